// Host side of the decode engine and the C ABI of include/qwen_cuda.h.
//
// An engine owns, on one GPU:
//   * every weight tensor in the device layout of common.cuh (one allocation);
//   * the fp32 KV cache, [layer][kv head][position][head_dim] (K and V);
//   * scratch activations, the RoPE table and the step state;
//   * a CUDA graph holding the kernels of one token step (decode.cu), replayed
//     once per token.
// It replaces reference src/model.rs Model (config, KV cache, forward) and the
// Backend of src/backend.rs for a whole token at a time.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <math.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstddef>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/qwen_cuda.h"
#include "gguf.h"
#include "kernels.h"
#include "layout.h"

namespace {

thread_local std::string g_last_error;

struct ApiError : std::runtime_error {
  int code;
  ApiError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define QC_CK(call)                                                                                        \
  do {                                                                                                     \
    cudaError_t e_ = (call);                                                                               \
    if (e_ != cudaSuccess)                                                                                 \
      throw ApiError(e_ == cudaErrorMemoryAllocation ? QC_ERR_NOMEM : QC_ERR_CUDA,                         \
                     std::string(#call) + ": " + cudaGetErrorString(e_));                                  \
  } while (0)

void ensure(bool c, const std::string& m, int code = QC_ERR_INVALID) {
  if (!c) throw ApiError(code, m);
}

constexpr uint64_t kChunk = 256ull << 20;  // staging size for weight upload
constexpr int kMaxSmem = 200 * 1024;

// One-time per-device kernel attributes.
void prepare_device(int device) {
  static std::mutex mu;
  static bool done[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= 64 || done[device]) return;
  QC_CK(qc::matvec_prepare(kMaxSmem));
  QC_CK(qc::decode_prepare(kMaxSmem));
  QC_CK(qc::token_prepare(0));
  QC_CK(qc::sample_prepare());
  QC_CK(qc::batch_prepare(kMaxSmem));
  QC_CK(qc::qgemm_prepare());
  done[device] = true;
}

struct TensorIn {
  std::string name;
  uint32_t kind = 0;
  std::vector<uint64_t> dims;
  const uint8_t* data = nullptr;
  uint64_t len = 0;
};

uint64_t align256(uint64_t v) { return (v + 255) & ~255ull; }

// Device placement of one tensor (8-row-group layout) and, for vectors, an f32 copy.
struct Placed {
  const TensorIn* t = nullptr;
  uint64_t rows = 1, experts = 1, cols = 0;
  uint64_t src_off = 0;  // byte offset of the first uploaded row in the tensor (expert shards)
  qc::DevLayout lay;
  uint64_t off = 0, off_f32 = 0;
  bool vector = false;
};

// Uploads raw GGUF rows to the device layout through double-buffered staging.
class Uploader {
 public:
  // Staging holds at least one row and at most max(kChunk, one row); `total` caps it for small uploads.
  Uploader(cudaStream_t s, uint64_t max_row, uint64_t total = kChunk) : s_(s) {
    uint64_t n = total < kChunk ? total : kChunk;
    n = max_row > n ? max_row : n;
    QC_CK(cudaMalloc(&buf_[0], n));
    QC_CK(cudaMalloc(&buf_[1], n));
    cap_ = n;
  }
  ~Uploader() {
    cudaStreamSynchronize(s_);
    cudaFree(buf_[0]);
    cudaFree(buf_[1]);
  }
  // `n_rows` raw rows (all experts, expert-major; `rows` per expert) of `raw_row` bytes
  // from host `src`, repacked into the 8-row-group layout at dst.
  uint64_t put(const uint8_t* src, uint64_t n_rows, uint32_t rows, uint64_t raw_row, uint32_t kind, uint64_t cols,
               uint8_t* dst, const qc::DevLayout& lay, uint64_t expert_stride) {
    const uint64_t per = cap_ / raw_row;
    uint64_t done = 0;
    while (done < n_rows) {
      const uint64_t n = n_rows - done < per ? n_rows - done : per;
      uint8_t* b = buf_[k_++ & 1];
      QC_CK(cudaMemcpyAsync(b, src + done * raw_row, n * raw_row, cudaMemcpyHostToDevice, s_));
      qc::launch_repack(b, done, n, rows, raw_row, kind, cols, dst, lay, expert_stride, s_);
      QC_CK(cudaGetLastError());
      done += n;
    }
    return n_rows * raw_row;
  }

 private:
  cudaStream_t s_;
  uint8_t* buf_[2] = {nullptr, nullptr};
  uint64_t cap_ = 0;
  unsigned k_ = 0;
};

qc::MatDesc desc_of(uint32_t kind, uint64_t rows, uint64_t cols, const qc::DevLayout& lay, const uint8_t* w) {
  qc::MatDesc m{};
  m.w = w;
  m.kind = kind;
  m.rows = (uint32_t)rows;
  m.cols = (uint32_t)cols;
  m.units = lay.units;
  m.lpr = lay.lpr;
  m.upl = lay.upl;
  m.main_bytes = (uint32_t)lay.main_bytes;
  m.d_bytes = (uint32_t)lay.d_bytes;
  m.group_bytes = (uint32_t)lay.group_bytes;
  m.expert_stride = lay.expert_bytes(rows);
  return m;
}
qc::MatDesc make_desc(const Placed& p, uint8_t* base) {
  return desc_of(p.t->kind, p.rows, p.cols, p.lay, base + p.off);
}

// Same matrix, processed with `lpr` lanes per row (a power of two dividing units).
qc::MatDesc with_lpr(qc::MatDesc m, uint32_t lpr) {
  m.lpr = lpr;
  m.upl = m.units / lpr;
  return m;
}

}  // namespace

// sampling.rs:3-8 Sampler: parameters and the StdRng state, resident on one device.
struct qc_sampler {
  int device = 0;
  uint32_t top_k = 0;
  qc::SamplerDev* d = nullptr;
  uint32_t* h = nullptr;  // pinned: [0] err, [1] token
  cudaStream_t own = nullptr;
  void* scratch = nullptr;  // sort and fold arrays of sets larger than shared memory
  uint32_t scratch_n = 0;
  ~qc_sampler() {
    cudaSetDevice(device);
    if (own) cudaStreamDestroy(own);
    cudaFreeHost(h);
    cudaFree(d);
    cudaFree(scratch);
  }
  // Scratch for a sample over n ids (none when the top-k set fits the kernel's shared memory);
  // allocated before the first such sample and kept for later ones.
  qc::SampleScratch scratch_for(uint32_t n) {
    const uint32_t set = top_k > 0 && top_k < n ? top_k : n;
    if (set <= qc::sample_exact_max()) return qc::SampleScratch{};
    if (n > scratch_n) {
      QC_CK(cudaDeviceSynchronize());  // an earlier sample may still use the old arrays
      cudaFree(scratch);
      scratch = nullptr;
      scratch_n = 0;
      QC_CK(cudaMalloc(&scratch, qc::sample_scratch_bytes(n)));
      scratch_n = n;
    }
    return qc::sample_scratch_at(scratch, n);
  }
  // Reads the sampled id and the sticky error after `st` drains; the error is cleared.
  uint32_t finish(cudaStream_t st) {
    static_assert(offsetof(qc::SamplerDev, token) == offsetof(qc::SamplerDev, err) + 4, "err, token adjacent");
    QC_CK(cudaMemcpyAsync(h, &d->err, 8, cudaMemcpyDeviceToHost, st));
    QC_CK(cudaStreamSynchronize(st));
    if (h[0]) {
      QC_CK(cudaMemsetAsync(&d->err, 0, 4, st));
      QC_CK(cudaStreamSynchronize(st));
      throw ApiError(QC_ERR_INVALID, "invalid logits");
    }
    return h[1];
  }
};

struct qc_engine {
  int device = 0, sms = 148;
  qc_config cfg{};
  uint32_t context = 0;
  uint8_t* d_weights = nullptr;
  uint64_t weight_bytes = 0;
  float* d_kv = nullptr;
  uint64_t kv_bytes = 0;
  uint8_t* d_scratch = nullptr;
  qc::DevState* d_state = nullptr;
  qc::DevState h_template{};
  std::vector<qc::LayerDev> layers;
  qc::MatDesc embd{}, out{};
  const float* out_norm = nullptr;
  qc::Scratch sc{};
  qc::DecodeDims dims{};
  qc::StepPlan plan{};
  // whole-token kernel: its plan, exchange buffers and the device copy of `layers`
  qc::TokenPlan tplan{};
  const char* token_why = nullptr;  // why the model does not fit it (nullptr: it fits)
  unsigned long long* d_ll = nullptr;
  qc::LayerDev* d_layers = nullptr;
  bool use_token = false;
  // expert parallelism: this engine holds experts [e_lo, e_lo + e_n) of `ep_world` shards and adds its
  // partial MoE vector into the peers' exchange buffers (CUDA IPC mappings)
  uint32_t ep_rank = 0, ep_world = 1, e_lo = 0, e_n = 0;
  bool ep_connected = false;
  unsigned long long* peer_ll[8] = {};
  unsigned long long** d_peers = nullptr;
  uint32_t* d_gen = nullptr;
  cudaStream_t own = nullptr, stream = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  uint32_t* h_pinned = nullptr;  // [0] token, [2..3] flags, then gen_count/cap
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  uint32_t pos = 0;
  qc_stats stats{};
  std::string err;

  ~qc_engine() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    if (exec) cudaGraphExecDestroy(exec);
    if (prof_exec) cudaGraphExecDestroy(prof_exec);
    if (prof_graph) cudaGraphDestroy(prof_graph);
    for (cudaEvent_t ev : prof_ev) cudaEventDestroy(ev);
    if (graph) cudaGraphDestroy(graph);
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    if (h_pinned) cudaFreeHost(h_pinned);
    cudaFree(d_weights);
    cudaFree(d_kv);
    cudaFree(d_scratch);
    for (uint32_t q = 0; q < ep_world && q < 8; q++)
      if (q != ep_rank && peer_ll[q]) cudaIpcCloseMemHandle(peer_ll[q]);
    cudaFree(d_peers);
    cudaFree(d_ll);
    cudaFree(d_moe);
    cudaFree(d_gemm);
    cudaFree(d_layers);
    if (own) cudaStreamDestroy(own);
  }

  // ---- model.rs:58-149: config and tensor validation -------------------------------------
  static void validate_config(const qc_config& c) {
    ensure(c.hidden > 0 && c.layers > 0 && c.layers <= 256 && c.kvheads > 0 && c.heads > 0 &&
               c.heads % c.kvheads == 0 && c.head_dim > 0 && c.head_dim % 2 == 0 && c.top > 0 &&
               c.top <= c.experts && c.experts <= 1024 && c.intermediate > 0 && std::isfinite(c.eps) && c.eps > 0.f &&
               std::isfinite(c.theta) && c.theta > 0.f,
           "invalid Qwen3 MoE config");
    // limits of this engine's kernels (shared-memory tiles), beyond the reference's own checks
    ensure(c.head_dim <= 256 && c.head_dim % 4 == 0, "the CUDA engine needs head_dim a multiple of 4, at most 256");
    ensure(c.heads / c.kvheads <= 64 && c.kvheads <= 64, "more than 64 query heads per KV head or KV heads");
    ensure(c.top <= 64, "more than 64 experts per token is not supported by the CUDA engine");
    ensure(c.hidden <= 8192, "hidden size above 8192 is not supported by the CUDA engine");
  }

  void check_shape(const std::map<std::string, TensorIn>& t, const std::string& n, std::vector<uint64_t> shape) {
    auto it = t.find(n);
    ensure(it != t.end(), "missing tensor " + n);
    ensure(it->second.dims == shape, n + ": unexpected shape");
  }

  void validate_tensors(const std::map<std::string, TensorIn>& t) {
    const qc_config& c = cfg;
    check_shape(t, "token_embd.weight", {c.hidden, c.vocab});
    check_shape(t, "output_norm.weight", {c.hidden});
    if (t.count("output.weight")) check_shape(t, "output.weight", {c.hidden, c.vocab});
    for (uint32_t i = 0; i < c.layers; i++) {
      const std::string b = "blk." + std::to_string(i) + ".";
      check_shape(t, b + "attn_norm.weight", {c.hidden});
      check_shape(t, b + "ffn_norm.weight", {c.hidden});
      check_shape(t, b + "attn_q_norm.weight", {c.head_dim});
      check_shape(t, b + "attn_k_norm.weight", {c.head_dim});
      check_shape(t, b + "attn_q.weight", {c.hidden, (uint64_t)c.heads * c.head_dim});
      check_shape(t, b + "attn_k.weight", {c.hidden, (uint64_t)c.kvheads * c.head_dim});
      check_shape(t, b + "attn_v.weight", {c.hidden, (uint64_t)c.kvheads * c.head_dim});
      check_shape(t, b + "attn_output.weight", {(uint64_t)c.heads * c.head_dim, c.hidden});
      check_shape(t, b + "ffn_gate_inp.weight", {c.hidden, c.experts});
      check_shape(t, b + "ffn_gate_exps.weight", {c.hidden, c.intermediate, c.experts});
      check_shape(t, b + "ffn_up_exps.weight", {c.hidden, c.intermediate, c.experts});
      check_shape(t, b + "ffn_down_exps.weight", {c.intermediate, c.hidden, c.experts});
      for (auto& kv : t) {
        const std::string& n = kv.first;
        const bool bias = n.size() >= 5 && n.compare(n.size() - 5, 5, ".bias") == 0;
        ensure(!(n.rfind(b, 0) == 0 && bias), "unexpected bias tensors");
      }
    }
  }

  // ---- build ------------------------------------------------------------------------------
  void build(const std::map<std::string, TensorIn>& t, const qc_config& c, uint32_t ctx, int dev, uint32_t rank = 0,
             uint32_t world = 1) {
    cfg = c;
    validate_config(cfg);
    validate_tensors(t);
    ensure(world >= 1 && world <= 8 && rank < world, "expert parallelism: need 1 <= world <= 8 and rank < world");
    ensure(cfg.experts % world == 0, "expert parallelism: the expert count must be a multiple of the world size");
    ep_rank = rank;
    ep_world = world;
    e_n = cfg.experts / world;
    e_lo = rank * e_n;
    ensure(ctx > 0 && ctx <= cfg.max_context, "context must be in 1..=" + std::to_string(cfg.max_context));
    context = ctx;
    device = dev;
    QC_CK(cudaSetDevice(device));
    cudaDeviceProp prop;
    QC_CK(cudaGetDeviceProperties(&prop, device));
    sms = prop.multiProcessorCount;
    prepare_device(device);
    QC_CK(cudaStreamCreateWithFlags(&own, cudaStreamNonBlocking));
    stream = own;

    // placement of every tensor the forward reads
    std::vector<std::string> names = {"token_embd.weight", "output_norm.weight"};
    const bool tied = !t.count("output.weight");
    if (!tied) names.push_back("output.weight");
    static const char* per_layer[] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_q_norm", "attn_k_norm",
                                      "attn_output", "ffn_norm", "ffn_gate_inp", "ffn_gate_exps", "ffn_up_exps",
                                      "ffn_down_exps"};
    for (uint32_t i = 0; i < cfg.layers; i++)
      for (const char* n : per_layer) names.push_back("blk." + std::to_string(i) + "." + n + ".weight");
    std::map<std::string, Placed> placed;
    uint64_t off = 0, max_row = 0;
    for (const std::string& n : names) {
      const TensorIn& ti = t.at(n);
      Placed p;
      p.t = &ti;
      p.cols = ti.dims[0];
      p.rows = ti.dims.size() > 1 ? ti.dims[1] : 1;
      p.experts = ti.dims.size() > 2 ? ti.dims[2] : 1;
      p.vector = ti.dims.size() == 1;
      uint64_t raw_row;
      if (const char* e = qc::ggml_row_bytes(ti.kind, p.cols, &raw_row)) throw ApiError(QC_ERR_INVALID, n + ": " + e);
      ensure(ti.len == raw_row * p.rows * p.experts, n + ": tensor length does not match its shape");
      if (p.experts > 1) {  // an expert stack: only this shard's experts are placed and uploaded
        p.src_off = (uint64_t)e_lo * p.rows * raw_row;
        p.experts = e_n;
      }
      ensure(p.rows <= 0xffffffffull && p.cols <= 0xffffffffull, n + ": tensor too large");
      max_row = raw_row > max_row ? raw_row : max_row;
      p.lay = qc::dev_layout(ti.kind, p.cols);
      ensure(p.lay.group_bytes <= 0xffffffffull, n + ": rows too wide");
      p.off = off;
      off = align256(off + p.lay.expert_bytes(p.rows) * p.experts);
      if (p.vector) {
        p.off_f32 = off;
        off = align256(off + p.cols * sizeof(float));
      }
      placed[n] = p;
    }
    weight_bytes = off;
    QC_CK(cudaMalloc(&d_weights, weight_bytes));
    QC_CK(cudaMemsetAsync(d_weights, 0, weight_bytes, stream));  // padding rows and blocks read as zero
    {
      Uploader up(stream, max_row);
      for (const std::string& n : names) {
        const Placed& p = placed[n];
        uint64_t raw_row;
        qc::ggml_row_bytes(p.t->kind, p.cols, &raw_row);
        stats.uploaded_bytes += up.put(p.t->data + p.src_off, p.rows * p.experts, (uint32_t)p.rows, raw_row, p.t->kind,
                                       p.cols, d_weights + p.off, p.lay, p.lay.expert_bytes(p.rows));
        if (p.vector) {
          qc::launch_dequant(make_desc(p, d_weights), 0, reinterpret_cast<float*>(d_weights + p.off_f32), stream);
          QC_CK(cudaGetLastError());
        }
      }
      QC_CK(cudaStreamSynchronize(stream));
    }
    auto vec = [&](const std::string& n) { return reinterpret_cast<const float*>(d_weights + placed[n].off_f32); };
    embd = make_desc(placed["token_embd.weight"], d_weights);
    out = tied ? embd : make_desc(placed["output.weight"], d_weights);
    out_norm = vec("output_norm.weight");

    // KV cache: [layer][kvhead][ctx][D], K then V
    const uint64_t D = cfg.head_dim, per_layer_kv = (uint64_t)cfg.kvheads * context * D;
    kv_bytes = per_layer_kv * cfg.layers * 2 * sizeof(float);
    QC_CK(cudaMalloc(&d_kv, kv_bytes));
    layers.resize(cfg.layers);
    for (uint32_t i = 0; i < cfg.layers; i++) {
      const std::string b = "blk." + std::to_string(i) + ".";
      qc::LayerDev& L = layers[i];
      L.q = make_desc(placed[b + "attn_q.weight"], d_weights);
      L.k = make_desc(placed[b + "attn_k.weight"], d_weights);
      L.v = make_desc(placed[b + "attn_v.weight"], d_weights);
      uint32_t lpr = L.q.lpr < L.k.lpr ? L.q.lpr : L.k.lpr;
      lpr = lpr < L.v.lpr ? lpr : L.v.lpr;
      L.q = with_lpr(L.q, lpr);
      L.k = with_lpr(L.k, lpr);
      L.v = with_lpr(L.v, lpr);
      L.o = make_desc(placed[b + "attn_output.weight"], d_weights);
      L.router = make_desc(placed[b + "ffn_gate_inp.weight"], d_weights);
      L.gate = make_desc(placed[b + "ffn_gate_exps.weight"], d_weights);
      L.up = make_desc(placed[b + "ffn_up_exps.weight"], d_weights);
      const uint32_t lg = L.gate.lpr < L.up.lpr ? L.gate.lpr : L.up.lpr;
      L.gate = with_lpr(L.gate, lg);
      L.up = with_lpr(L.up, lg);
      L.down = make_desc(placed[b + "ffn_down_exps.weight"], d_weights);
      L.attn_norm = vec(b + "attn_norm.weight");
      L.q_norm = vec(b + "attn_q_norm.weight");
      L.k_norm = vec(b + "attn_k_norm.weight");
      L.ffn_norm = vec(b + "ffn_norm.weight");
      L.kc = d_kv + (uint64_t)i * 2 * per_layer_kv;
      L.vc = L.kc + per_layer_kv;
    }

    // scratch
    dims.hidden = cfg.hidden;
    dims.heads = cfg.heads;
    dims.kvheads = cfg.kvheads;
    dims.head_dim = cfg.head_dim;
    dims.experts = cfg.experts;
    dims.top = cfg.top;
    dims.inter = cfg.intermediate;
    dims.vocab = cfg.vocab;
    dims.ctx = context;
    dims.eps = cfg.eps;
    uint32_t nsplit = 32;
    while ((context + nsplit - 1) / nsplit > 128) nsplit *= 2;
    dims.nsplit = nsplit;
    const uint64_t G = cfg.heads / cfg.kvheads, QD = (uint64_t)cfg.heads * D, KD = (uint64_t)cfg.kvheads * D;
    uint64_t so = 0;
    auto take = [&](uint64_t bytes) {
      const uint64_t o = so;
      so = align256(so + bytes);
      return o;
    };
    const uint64_t o_x = take(cfg.hidden * 4), o_qkv = take((QD + 2 * KD) * 4);
    const uint64_t o_attn = take(QD * 4), o_part = take((uint64_t)cfg.kvheads * nsplit * G * (D + 2) * 4);
    const uint64_t o_rl = take(cfg.experts * 4), o_sel = take(cfg.top * 4), o_selw = take(cfg.top * 4);
    const uint64_t o_h = take((uint64_t)cfg.top * cfg.intermediate * 4), o_log = take((uint64_t)cfg.vocab * 4);
    const uint64_t o_rope = take((uint64_t)context * (D / 2) * 8), o_gen = take((uint64_t)context * 4);
    const uint64_t o_st = take(sizeof(qc::DevState));
    QC_CK(cudaMalloc(&d_scratch, so));
    QC_CK(cudaMemsetAsync(d_scratch, 0, so, stream));
    sc.x = reinterpret_cast<float*>(d_scratch + o_x);
    sc.qkv = reinterpret_cast<float*>(d_scratch + o_qkv);
    sc.attn = reinterpret_cast<float*>(d_scratch + o_attn);
    sc.part = reinterpret_cast<float*>(d_scratch + o_part);
    sc.rlogit = reinterpret_cast<float*>(d_scratch + o_rl);
    sc.sel = reinterpret_cast<uint32_t*>(d_scratch + o_sel);
    sc.selw = reinterpret_cast<float*>(d_scratch + o_selw);
    sc.h = reinterpret_cast<float*>(d_scratch + o_h);
    sc.logits = reinterpret_cast<float*>(d_scratch + o_log);
    sc.rope = reinterpret_cast<const float2*>(d_scratch + o_rope);
    d_gen = reinterpret_cast<uint32_t*>(d_scratch + o_gen);
    d_state = reinterpret_cast<qc::DevState*>(d_scratch + o_st);

    // RoPE angles exactly as ops.rs:17-28 computes them on the host: pos * theta^(-2i/D) in f32.
    std::vector<float2> rope((uint64_t)context * (D / 2));
    for (uint64_t p = 0; p < context; p++)
      for (uint64_t i = 0; i < D / 2; i++) {
        const float e = -2.0f * (float)i / (float)D;
        const float angle = (float)p * powf(cfg.theta, e);
        rope[p * (D / 2) + i] = make_float2(cosf(angle), sinf(angle));
      }
    QC_CK(cudaMemcpyAsync(d_scratch + o_rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice,
                          stream));
    h_template = qc::DevState{};
    h_template.seq = 1;  // exchange buffers start at tag 0
    h_template.gen_tokens = d_gen;
    h_template.gen_cap = context;
    QC_CK(cudaMemcpyAsync(d_state, &h_template, sizeof h_template, cudaMemcpyHostToDevice, stream));
    QC_CK(cudaMallocHost(&h_pinned, 64));
    QC_CK(cudaEventCreate(&ev0));
    QC_CK(cudaEventCreate(&ev1));
    QC_CK(cudaStreamSynchronize(stream));
    QC_CK(cudaMalloc(&d_layers, layers.size() * sizeof(qc::LayerDev)));
    QC_CK(cudaMemcpy(d_layers, layers.data(), layers.size() * sizeof(qc::LayerDev), cudaMemcpyHostToDevice));
    plan = qc::plan_step(step_args());
    ensure(qc::step_smem_max(step_args(), plan) <= (size_t)kMaxSmem,
           "model dimensions need more shared memory per block than the CUDA engine supports");
    token_why = qc::plan_token(step_args(), 1 << 30, &tplan);
    ensure(world == 1 || !token_why,
           std::string("expert parallelism needs the whole-token kernel: ") + (token_why ? token_why : ""));
    QC_CK(cudaMalloc(&d_peers, 8 * sizeof(unsigned long long*)));
    if (!token_why) {
      const uint64_t n = tplan.ll_layer * cfg.layers;
      QC_CK(cudaMalloc(&d_ll, n * sizeof(unsigned long long)));
      QC_CK(cudaMemset(d_ll, 0, n * sizeof(unsigned long long)));  // tag 0: never a token's tag
    }
    use_token = !token_why;
    ep_connected = world == 1;
    if (world == 1) {
      peer_ll[0] = d_ll;
      QC_CK(cudaMemcpy(d_peers, peer_ll, 8 * sizeof(unsigned long long*), cudaMemcpyHostToDevice));
      capture();
    }
  }

  qc::StepArgs step_args() const {
    qc::StepArgs a{};
    a.dims = dims;
    a.sc = sc;
    a.st = d_state;
    a.layers = layers.data();
    a.layers_dev = d_layers;
    a.n_layers = cfg.layers;
    a.ep_rank = ep_rank;
    a.ep_world = ep_world;
    a.e_lo = e_lo;
    a.e_n = e_n;
    a.peers = d_peers;
    a.embd = embd;
    a.out = out;
    a.out_norm = out_norm;
    a.sms = sms;
    return a;
  }

  void capture() {
    if (use_token) {  // a device or driver that cannot capture the cooperative launch keeps the per-phase kernels
      try {
        capture_once();
        return;
      } catch (const ApiError&) {
        if (ep_world > 1) throw;  // the per-phase kernels have no expert-parallel form
        cudaGetLastError();
        token_why = "the cooperative whole-token launch could not be captured in a CUDA graph";
        use_token = false;
      }
    }
    capture_once();
  }

  void capture_once() {
    cudaStream_t cs;
    QC_CK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    QC_CK(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    if (use_token) qc::launch_token(step_args(), tplan, d_ll, true, cs);
    else qc::launch_step(step_args(), plan, cs);
    cudaError_t le = cudaGetLastError();
    cudaError_t ce = cudaStreamEndCapture(cs, &graph);
    cudaStreamDestroy(cs);
    QC_CK(le);
    QC_CK(ce);
    QC_CK(cudaGraphInstantiate(&exec, graph, 0));
  }

  // Decode path: 0 = the whole-token kernel when the model fits it, 1 = the per-phase kernels.
  void set_mode(int mode) {
    ensure(mode == 0 || mode == 1, "decode mode must be 0 (auto) or 1 (per-phase kernels)");
    ensure(mode == 0 || ep_world == 1, "an expert-parallel engine runs only the whole-token kernel");
    const bool want = mode == 0 && !token_why;
    if (want == use_token) return;
    QC_CK(cudaSetDevice(device));
    QC_CK(cudaStreamSynchronize(stream));
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    exec = nullptr;
    graph = nullptr;
    if (prof_exec) cudaGraphExecDestroy(prof_exec);
    if (prof_graph) cudaGraphDestroy(prof_graph);
    prof_exec = nullptr;
    prof_graph = nullptr;
    for (cudaEvent_t ev : prof_ev) cudaEventDestroy(ev);
    prof_ev.clear();
    prof_kind.clear();
    use_token = want;
    capture();
  }

  // ---- expert parallelism: exchange-buffer handles -------------------------------------------
  void ep_handle(void* out_handle, int* pci) {
    ensure(ep_world > 1, "not an expert-parallel engine");
    QC_CK(cudaSetDevice(device));
    cudaIpcMemHandle_t h;
    QC_CK(cudaIpcGetMemHandle(&h, d_ll));
    std::memcpy(out_handle, &h, sizeof h);
    cudaDeviceProp prop;
    QC_CK(cudaGetDeviceProperties(&prop, device));
    *pci = prop.pciDomainID * 65536 + prop.pciBusID * 256 + prop.pciDeviceID;
  }
  void ep_connect(const uint8_t* handles, const int* pci) {
    ensure(ep_world > 1, "not an expert-parallel engine");
    ensure(!ep_connected, "expert-parallel engine already connected");
    for (uint32_t a = 0; a < ep_world; a++)
      for (uint32_t b = a + 1; b < ep_world; b++)
        ensure(pci[a] != pci[b], "expert-parallel ranks must be on different GPUs");  // kernels wait on each other
    QC_CK(cudaSetDevice(device));
    for (uint32_t q = 0; q < ep_world; q++) {
      if (q == ep_rank) {
        peer_ll[q] = d_ll;
        continue;
      }
      cudaIpcMemHandle_t h;
      std::memcpy(&h, handles + 64 * q, sizeof h);
      void* ptr = nullptr;
      QC_CK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
      peer_ll[q] = static_cast<unsigned long long*>(ptr);
    }
    QC_CK(cudaMemcpy(d_peers, peer_ll, 8 * sizeof(unsigned long long*), cudaMemcpyHostToDevice));
    ep_connected = true;
    capture();
  }

  // ---- model.rs:202-216 ------------------------------------------------------------------
  void reset() {
    cudaSetDevice(device);
    // any earlier asynchronous failure is reported by the caller; the reset itself must not throw past here.
    // The token tag (DevState::seq, the last field) is kept.
    cudaMemcpyAsync(d_state, &h_template, offsetof(qc::DevState, seq), cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
    pos = 0;
  }

  // ---- per-kernel timing: a second graph with external event records between kernels ----
  cudaGraphExec_t prof_exec = nullptr;
  cudaGraph_t prof_graph = nullptr;
  std::vector<cudaEvent_t> prof_ev;
  std::vector<int> prof_kind;

  struct ProfCtx {
    qc_engine* e;
    cudaError_t err;
  };
  static void prof_hook(void* p, int kind, cudaStream_t s) {
    ProfCtx* c = static_cast<ProfCtx*>(p);
    qc_engine* e = c->e;
    cudaEvent_t ev;
    cudaError_t r = cudaEventCreate(&ev);
    if (r == cudaSuccess) r = cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal);
    if (r != cudaSuccess && c->err == cudaSuccess) c->err = r;
    e->prof_ev.push_back(ev);
    e->prof_kind.push_back(kind);
  }

  void profile(qc_phase_times* out) {
    ensure(pos < context, "context limit " + std::to_string(context) + " reached", QC_ERR_CONTEXT);
    ensure(ep_connected, "expert-parallel engine is not connected to its peers");
    QC_CK(cudaSetDevice(device));
    if (use_token) {  // one kernel per token: its whole duration
      *out = qc_phase_times{};
      QC_CK(cudaEventRecord(ev0, stream));
      QC_CK(cudaGraphLaunch(exec, stream));
      QC_CK(cudaEventRecord(ev1, stream));
      check_flags();
      float ms = 0.f;
      QC_CK(cudaEventElapsedTime(&ms, ev0, ev1));
      out->token_ms = ms;
      out->launches = 1;
      pos += 1;
      stats.tokens += 1;
      return;
    }
    if (!prof_exec) {
      cudaStream_t cs;
      QC_CK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
      ProfCtx ctx{this, cudaSuccess};
      QC_CK(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
      qc::launch_step(step_args(), plan, cs, &qc_engine::prof_hook, &ctx);
      cudaError_t le = cudaGetLastError();
      cudaError_t ce = cudaStreamEndCapture(cs, &prof_graph);
      cudaStreamDestroy(cs);
      QC_CK(ctx.err);
      QC_CK(le);
      QC_CK(ce);
      QC_CK(cudaGraphInstantiate(&prof_exec, prof_graph, 0));
    }
    QC_CK(cudaGraphLaunch(prof_exec, stream));
    check_flags();
    double* slot[qc::K_COUNT] = {&out->embed_ms, &out->attn_in_ms, &out->attention_ms, &out->oproj_ms,
                                 &out->router_ms, &out->gateup_ms, &out->down_ms, &out->output_ms};
    *out = qc_phase_times{};
    for (size_t i = 0; i + 1 < prof_ev.size(); i++) {
      float ms = 0.f;
      QC_CK(cudaEventElapsedTime(&ms, prof_ev[i], prof_ev[i + 1]));
      *slot[prof_kind[i]] += ms;
      out->token_ms += ms;
    }
    out->launches = qc::step_launches(cfg.layers);
    pos += 1;
    stats.tokens += 1;
  }

  void launch_steps(uint32_t n) {
    for (uint32_t i = 0; i < n; i++) QC_CK(cudaGraphLaunch(exec, stream));
  }

  // Reads the sticky flags after `stream` is drained; a set flag is an error.
  void check_flags() {
    QC_CK(cudaMemcpyAsync(h_pinned + 2, &d_state->nonfinite, 8, cudaMemcpyDeviceToHost, stream));
    QC_CK(cudaMemcpyAsync(h_pinned + 6, &d_state->abort, 4, cudaMemcpyDeviceToHost, stream));
    QC_CK(cudaStreamSynchronize(stream));
    if (h_pinned[6]) throw ApiError(QC_ERR_CUDA, "decode kernel: a wait between thread blocks timed out");
    if (h_pinned[3]) throw ApiError(QC_ERR_TOKEN, "token outside vocabulary");
    if (h_pinned[2]) throw ApiError(QC_ERR_NONFINITE, "nonfinite model output");
  }

  void forward(uint32_t token, float* logits) {
    ensure(ep_connected, "expert-parallel engine is not connected to its peers");
    ensure(pos < context, "context limit " + std::to_string(context) + " reached", QC_ERR_CONTEXT);
    ensure(token < cfg.vocab, "token outside vocabulary", QC_ERR_TOKEN);
    QC_CK(cudaSetDevice(device));
    h_pinned[0] = token;
    QC_CK(cudaMemcpyAsync(&d_state->token, h_pinned, 4, cudaMemcpyHostToDevice, stream));
    QC_CK(cudaEventRecord(ev0, stream));
    launch_steps(1);
    QC_CK(cudaEventRecord(ev1, stream));
    if (logits) QC_CK(cudaMemcpyAsync(logits, sc.logits, (size_t)cfg.vocab * 4, cudaMemcpyDeviceToHost, stream));
    check_flags();
    float ms = 0.f;
    QC_CK(cudaEventElapsedTime(&ms, ev0, ev1));
    stats.matvec_ms += ms;
    stats.tokens += 1;
    stats.matvecs += (5ull + 3ull * cfg.top) * cfg.layers + 1;
    pos += 1;
  }

  void decode(uint32_t n, uint32_t* tokens_out, float* logits, bool wait) {
    ensure(ep_connected, "expert-parallel engine is not connected to its peers");
    ensure(pos > 0, "greedy decode needs the logits of a previous forward");
    ensure((uint64_t)pos + n <= context, "prompt + max-tokens exceed --ctx", QC_ERR_CONTEXT);
    QC_CK(cudaSetDevice(device));
    h_pinned[4] = 0;  // gen_count
    QC_CK(cudaMemcpyAsync(&d_state->gen_count, h_pinned + 4, 4, cudaMemcpyHostToDevice, stream));
    if (wait) QC_CK(cudaEventRecord(ev0, stream));
    launch_steps(n);
    pos += n;
    stats.tokens += n;
    stats.matvecs += ((5ull + 3ull * cfg.top) * cfg.layers + 1) * n;
    if (!wait) return;
    QC_CK(cudaEventRecord(ev1, stream));
    if (tokens_out && n) QC_CK(cudaMemcpyAsync(tokens_out, d_gen, (size_t)n * 4, cudaMemcpyDeviceToHost, stream));
    if (logits) QC_CK(cudaMemcpyAsync(logits, sc.logits, (size_t)cfg.vocab * 4, cudaMemcpyDeviceToHost, stream));
    check_flags();
    float ms = 0.f;
    QC_CK(cudaEventElapsedTime(&ms, ev0, ev1));
    stats.matvec_ms += ms;
  }

  // ---- the tensor-core GEMM's copy of the weights ---------------------------------------------
  uint8_t* d_gemm = nullptr;
  std::vector<qc::GemmMat> gemm;  // per layer: q, k, v, o, gate, up, down; then the output matrix (w null: none)

  // The GEMM-layout copy of every Q4_K / Q6_K matrix the tensor-core paths read (batched projections,
  // grouped experts, vocabulary rows), made once, on first use: each (64-row tile, super-block) block
  // contiguous, so that a GEMM stage is two bulk copies.
  void ensure_gemm() {
    if (d_gemm) return;
    QC_CK(cudaSetDevice(device));
    const uint32_t L = cfg.layers;
    std::vector<std::pair<const qc::MatDesc*, uint32_t>> mats;
    for (uint32_t l = 0; l < L; l++) {
      const qc::LayerDev& d = layers[l];
      for (const qc::MatDesc* m : {&d.q, &d.k, &d.v, &d.o}) mats.push_back({m, 1u});
      for (const qc::MatDesc* m : {&d.gate, &d.up, &d.down}) mats.push_back({m, e_n});
    }
    mats.push_back({&out, 1u});
    std::vector<uint64_t> off(mats.size(), ~0ull);
    uint64_t total = 0;
    for (size_t i = 0; i < mats.size(); i++)
      if (!qc::qgemm_supported(mats[i].first->kind, mats[i].first->cols)) {
        off[i] = total;
        total = align256(total + qc::gemm_bytes(*mats[i].first, mats[i].second));
      }
    gemm.assign(mats.size(), qc::GemmMat{});
    if (total == 0) return;
    QC_CK(cudaMalloc(&d_gemm, total));
    for (size_t i = 0; i < mats.size(); i++)
      if (off[i] != ~0ull) {
        gemm[i] = qc::gemm_mat(*mats[i].first, d_gemm + off[i]);
        qc::launch_qg_relayout(*mats[i].first, mats[i].second, gemm[i], stream);
      }
    QC_CK(cudaGetLastError());
    QC_CK(cudaStreamSynchronize(stream));
  }
  const qc::GemmMat& gm(uint32_t layer, uint32_t which) const { return gemm[7 * layer + which]; }

  // ---- the MoE half of one layer for a batch of tokens --------------------------------------
  uint8_t* d_moe = nullptr;  // scratch of moe_cap tokens
  uint32_t moe_cap = 0;
  std::vector<float> moe_sw;  // per layer: Q4_K min-block scales (gate, up, down); 0 = not yet measured

  qc::MoeArgs moe_args(uint32_t layer, uint32_t T) {
    const qc::LayerDev& L = layers[layer];
    qc::MoeArgs a{};
    a.router = L.router;
    a.gate = L.gate;
    a.up = L.up;
    a.down = L.down;
    if (!gemm.empty()) {
      a.ggate = gm(layer, 4);
      a.gup = gm(layer, 5);
      a.gdown = gm(layer, 6);
    }
    a.ffn_norm = L.ffn_norm;
    a.H = cfg.hidden;
    a.I = cfg.intermediate;
    a.E = cfg.experts;
    a.top = cfg.top;
    a.T = T;
    a.eps = cfg.eps;
    a.sms = sms;
    a.NPgu = a.NPdn = 8;
    a.SSgu = a.SSdn = 2;
    if (!qc::qgemm_shape(a.gate.kind, a.H, a.gate.kind == qc::Q4_K, &a.NPgu, &a.SSgu))
      qc::qgemm_shape(a.down.kind, a.I, a.down.kind == qc::Q4_K, &a.NPdn, &a.SSdn);
    const uint64_t P = (uint64_t)moe_cap * cfg.top, R = qc::moe_image_rows(moe_cap, cfg.top, cfg.experts);
    uint64_t o = 0;
    auto take = [&](uint64_t bytes) {
      uint8_t* p = d_moe + o;
      o = align256(o + bytes);
      return p;
    };
    a.h = reinterpret_cast<float*>(take((uint64_t)moe_cap * cfg.hidden * 4));
    a.hscale = reinterpret_cast<float*>(take(moe_cap * 4));
    a.rlg = reinterpret_cast<float*>(take((uint64_t)moe_cap * cfg.experts * 4));
    a.sel = reinterpret_cast<uint32_t*>(take(P * 4));
    a.selw = reinterpret_cast<float*>(take(P * 4));
    a.cnt = reinterpret_cast<uint32_t*>(take(cfg.experts * 4));
    a.off = reinterpret_cast<uint32_t*>(take(cfg.experts * 4));
    a.ptok = reinterpret_cast<uint32_t*>(take(P * 4));
    a.ppair = reinterpret_cast<uint32_t*>(take(P * 4));
    a.groups = reinterpret_cast<qc::QgGroup*>(take(2ull * cfg.experts * sizeof(qc::QgGroup)));
    a.nitems = reinterpret_cast<uint32_t*>(take(8));
    a.imgrows = reinterpret_cast<uint4*>(take(R * 16));
    a.nrows = reinterpret_cast<uint32_t*>(take(4));
    a.img_gu = take(R * qc::qg_image_row_bytes(cfg.hidden, a.gate.kind == qc::Q4_K));
    a.img_dn = take(R * qc::qg_image_row_bytes(cfg.intermediate, a.down.kind == qc::Q4_K));
    a.y = reinterpret_cast<float*>(take(P * cfg.hidden * 4));
    a.err = reinterpret_cast<uint32_t*>(take(4));
    // inputs and outputs of the call follow the scratch
    return a;
  }
  uint64_t moe_bytes(uint32_t cap) const {
    const uint64_t P = (uint64_t)cap * cfg.top, R = qc::moe_image_rows(cap, cfg.top, cfg.experts);
    auto al = [](uint64_t b) { return align256(b); };
    // (an upper bound: image rows are sized for Q4_K min chunks whatever the layer's formats)
    return al((uint64_t)cap * cfg.hidden * 4) + al(cap * 4) + al((uint64_t)cap * cfg.experts * 4) + 2 * al(P * 4) + 2 * al(cfg.experts * 4) +
           2 * al(P * 4) + al(2ull * cfg.experts * sizeof(qc::QgGroup)) + al(8) + al(R * 16) + al(4) +
           al(R * qc::qg_image_row_bytes(cfg.hidden, true)) + al(R * qc::qg_image_row_bytes(cfg.intermediate, true)) +
           al(P * cfg.hidden * 4) + al(4) + 2 * al((uint64_t)cap * cfg.hidden * 4);
  }

  // x, out: [T][hidden] host arrays.  path 1: the per-token decode kernels (router, gate/up, down)
  // once per token; path 2: the batched tensor-core kernels.  *ms: device time of the layer.
  // The MoE scratch (moe_args) for at least T tokens.
  void grow_moe(uint32_t T) {
    if (T <= moe_cap) return;
    QC_CK(cudaStreamSynchronize(stream));
    cudaFree(d_moe);
    d_moe = nullptr;
    moe_cap = 0;
    QC_CK(cudaMalloc(&d_moe, moe_bytes(T)));
    moe_cap = T;
  }
  // Power-of-two scales of the Q4_K min blocks of the tensor-core GEMM for a layer (from the largest
  // |dmin| of each expert stack, measured once per layer), into a.smin_g / smin_u / smin_d.
  void moe_scales(uint32_t layer, qc::MoeArgs& a) {
    if (moe_sw.empty()) moe_sw.assign(3 * cfg.layers, 0.f);
    if (moe_sw[3 * layer] == 0.f) {
      const qc::MatDesc* m[3] = {&a.gate, &a.up, &a.down};
      for (int i = 0; i < 3; i++) moe_sw[3 * layer + i] = dmin_scale(*m[i], e_n, a.err);
    }
    a.smin_g = moe_sw[3 * layer];
    a.smin_u = moe_sw[3 * layer + 1];
    a.smin_d = moe_sw[3 * layer + 2];
  }
  // Q4_K: 2^k with (largest |dmin|) * 63 * 2^k < 2^14 (the min block's fp16 hi/lo split); others 1.
  // `tmp` is one word of device scratch.
  float dmin_scale(const qc::MatDesc& m, uint32_t experts, uint32_t* tmp) {
    if (m.kind != qc::Q4_K) return 1.f;
    uint32_t hb = 0;
    QC_CK(cudaMemsetAsync(tmp, 0, 4, stream));
    qc::launch_qg_dmin(m, experts, tmp, stream);
    QC_CK(cudaMemcpyAsync(&hb, tmp, 4, cudaMemcpyDeviceToHost, stream));
    QC_CK(cudaMemsetAsync(tmp, 0, 4, stream));
    QC_CK(cudaStreamSynchronize(stream));
    float dmax;
    std::memcpy(&dmax, &hb, 4);
    return qc::qg_pow2_scale(dmax * 63.f);
  }

  void moe_layer(uint32_t layer, const float* x, uint32_t T, float* out, int path, float* ms) {
    ensure(layer < cfg.layers, "layer index out of range");
    ensure(T > 0 && x && out, "empty batch");
    ensure(path == 1 || path == 2, "MoE path must be 1 (per-token kernels) or 2 (tensor cores)");
    ensure(ep_world == 1, "an expert-parallel engine holds only its own experts");
    QC_CK(cudaSetDevice(device));
    if (path == 2) ensure_gemm();
    grow_moe(T);
    qc::MoeArgs a = moe_args(layer, T);
    const uint64_t xbytes = (uint64_t)T * cfg.hidden * 4;
    float* d_x = reinterpret_cast<float*>(d_moe + moe_bytes(moe_cap) - 2 * align256((uint64_t)moe_cap * cfg.hidden * 4));
    float* d_out = d_x + align256((uint64_t)moe_cap * cfg.hidden * 4) / 4;
    QC_CK(cudaMemcpyAsync(d_x, x, xbytes, cudaMemcpyHostToDevice, stream));
    if (path == 2) {
      if (const char* why = qc::moe_tc_supported(a)) throw ApiError(QC_ERR_INVALID, why);
      moe_scales(layer, a);
      QC_CK(cudaMemsetAsync(a.err, 0, 4, stream));
      QC_CK(cudaEventRecord(ev0, stream));
      if (const char* why = qc::launch_moe_tc(a, d_x, d_out, stream)) throw ApiError(QC_ERR_CUDA, why);
      QC_CK(cudaGetLastError());
      QC_CK(cudaEventRecord(ev1, stream));
      uint32_t herr = 0;
      QC_CK(cudaMemcpyAsync(&herr, a.err, 4, cudaMemcpyDeviceToHost, stream));
      QC_CK(cudaStreamSynchronize(stream));
      if (herr & 2) throw ApiError(QC_ERR_CUDA, "MoE tensor-core kernel: a wait timed out");
      if (herr & 1) throw ApiError(QC_ERR_NONFINITE, "non-finite router logits");
      if (herr & 4) throw ApiError(QC_ERR_NONFINITE, "an expert activation outside the fp16 range of the tensor-core path");
    } else {
      const qc::LayerDev& L = layers[layer];
      QC_CK(cudaEventRecord(ev0, stream));
      for (uint32_t t = 0; t < T; t++) {
        QC_CK(cudaMemcpyAsync(sc.x, d_x + (uint64_t)t * cfg.hidden, cfg.hidden * 4, cudaMemcpyDeviceToDevice, stream));
        qc::launch_moe_token(dims, plan, L, sc, d_state, stream);
        QC_CK(cudaGetLastError());
        QC_CK(cudaMemcpyAsync(d_out + (uint64_t)t * cfg.hidden, sc.x, cfg.hidden * 4, cudaMemcpyDeviceToDevice, stream));
      }
      QC_CK(cudaEventRecord(ev1, stream));
      QC_CK(cudaStreamSynchronize(stream));
      check_flags();
    }
    QC_CK(cudaMemcpyAsync(out, d_out, xbytes, cudaMemcpyDeviceToHost, stream));
    QC_CK(cudaStreamSynchronize(stream));
    float t_ms = 0.f;
    QC_CK(cudaEventElapsedTime(&t_ms, ev0, ev1));
    if (ms) *ms = t_ms;
  }

  // The chat loop with a sampler (main.rs:261-282): n times, sample the current logits on the
  // device and feed the id to the next step; tokens_out gets the n sampled ids.
  void decode_sample(qc_sampler* smp, uint32_t n, uint32_t* tokens_out, float* logits) {
    ensure(ep_connected, "expert-parallel engine is not connected to its peers");
    ensure(smp && smp->device == device, "the sampler lives on another device");
    ensure(pos > 0, "sampling needs the logits of a previous forward");
    ensure((uint64_t)pos + n <= context, "prompt + max-tokens exceed --ctx", QC_ERR_CONTEXT);
    QC_CK(cudaSetDevice(device));
    h_pinned[4] = 0;  // gen_count
    QC_CK(cudaMemcpyAsync(&d_state->gen_count, h_pinned + 4, 4, cudaMemcpyHostToDevice, stream));
    const qc::SampleScratch scr = smp->scratch_for(cfg.vocab);
    QC_CK(cudaEventRecord(ev0, stream));
    for (uint32_t i = 0; i < n; i++) {
      QC_CK(qc::launch_sample(sc.logits, cfg.vocab, smp->d, &d_state->token, scr, stream));
      launch_steps(1);
    }
    QC_CK(cudaEventRecord(ev1, stream));
    pos += n;
    stats.tokens += n;
    stats.matvecs += ((5ull + 3ull * cfg.top) * cfg.layers + 1) * n;
    if (tokens_out && n) QC_CK(cudaMemcpyAsync(tokens_out, d_gen, (size_t)n * 4, cudaMemcpyDeviceToHost, stream));
    if (logits) QC_CK(cudaMemcpyAsync(logits, sc.logits, (size_t)cfg.vocab * 4, cudaMemcpyDeviceToHost, stream));
    check_flags();
    smp->finish(stream);
    float ms = 0.f;
    QC_CK(cudaEventElapsedTime(&ms, ev0, ev1));
    stats.matvec_ms += ms;
  }
};

struct qc_matrix {
  int device = 0;
  qc::MatDesc desc{};
  uint8_t* d = nullptr;
  uint64_t bytes = 0, packed = 0, experts = 1;
  ~qc_matrix() {
    cudaSetDevice(device);
    cudaFree(d);
  }
};

// Several sequences decoded together (no counterpart in the reference, which runs
// one sequence): per-sequence KV caches beside an engine's weights, and one device pass per step for
// any mix of decode tokens and prompt chunks (batch.cu), with the MoE half on the tensor cores.
struct qc_batch {
  qc_engine* e = nullptr;
  uint32_t n_seqs = 0, context = 0, cap = 0;  // cap: tokens per device pass
  std::vector<uint32_t> pos;                  // next position of each sequence
  float* d_kv = nullptr;
  uint64_t kv_floats = 0;  // one K (or V) block of one layer of one sequence
  uint8_t* d_buf = nullptr;
  // pass scratch (cap tokens)
  qc::BatchTok* d_tok = nullptr;
  uint32_t* d_ids = nullptr;   // token ids of the pass
  uint32_t* d_osrc = nullptr;  // token index of each logits row of the pass
  float *d_x = nullptr, *d_x2 = nullptr, *d_q = nullptr, *d_k = nullptr, *d_v = nullptr, *d_a = nullptr;
  uint8_t* d_xv = nullptr;
  uint32_t xb_max = 0;
  float* d_lg = nullptr;     // [cap][vocab] logits rows of the pass
  // tensor-core projections (qgemm.cu): per layer, which of q, k, v, o take it and their Q4_K min
  // scales; the same for the vocabulary rows; the activation image and its vector scales
  std::vector<uint8_t> tc;     // [layer][4]
  std::vector<float> tc_smin;  // [layer][4]
  bool tc_out = false;
  float tc_out_smin = 1.f;
  uint8_t* d_img = nullptr;
  float* d_hs = nullptr;
  float* d_last = nullptr;   // [n_seqs][vocab] the latest logits of each sequence
  uint32_t* d_flag = nullptr;  // [0] non-finite logits
  // sampling
  const float** d_rows = nullptr;       // [n_seqs] logits rows of the draws
  qc::SamplerDev** d_sv = nullptr;      // [n_seqs] samplers of the draws
  uint32_t* d_out = nullptr;            // [n_seqs * out_cap] sampled ids of a decode loop
  uint32_t out_cap = 0;
  void* d_sscr = nullptr;               // [n_seqs] sample scratch (sets beyond shared memory)
  qc_stats stats{};
  std::string err;
  // expert parallelism (an engine holding experts/world of every layer): this rank's exchange region
  // (moe.cu MoeEp layout, two buffer sets), the peers' regions mapped by CUDA IPC, the barrier count
  // and the running layer count that picks the buffer set
  uint8_t* d_ep = nullptr;
  uint8_t* ep_peer[8] = {};
  uint8_t** d_ep_peers = nullptr;
  qc::MoeEp ep_set[2] = {};
  bool ep_connected = false, ep_failed = false;
  unsigned long long ep_seq = 0, ep_layers = 0;

  ~qc_batch() {
    cudaSetDevice(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    for (uint32_t q = 0; q < e->ep_world && q < 8; q++)
      if (q != e->ep_rank && ep_peer[q]) cudaIpcCloseMemHandle(ep_peer[q]);
    cudaFree(d_ep);
    cudaFree(d_ep_peers);
    cudaFree(d_kv);
    cudaFree(d_buf);
    cudaFree(d_out);
    cudaFree(d_sscr);
  }

  // ---- expert parallelism: exchange-region handles (as qc_engine's) ---------------------------
  void ep_handle(void* out_handle, int* pci) {
    ensure(e->ep_world > 1, "not an expert-parallel engine");
    QC_CK(cudaSetDevice(e->device));
    cudaIpcMemHandle_t h;
    QC_CK(cudaIpcGetMemHandle(&h, d_ep));
    std::memcpy(out_handle, &h, sizeof h);
    cudaDeviceProp prop;
    QC_CK(cudaGetDeviceProperties(&prop, e->device));
    *pci = prop.pciDomainID * 65536 + prop.pciBusID * 256 + prop.pciDeviceID;
  }
  void ep_connect(const uint8_t* handles, const int* pci) {
    const uint32_t W = e->ep_world, R = e->ep_rank;
    ensure(W > 1, "not an expert-parallel engine");
    ensure(!ep_connected, "expert-parallel batch already connected");
    for (uint32_t a = 0; a < W; a++)
      for (uint32_t b = a + 1; b < W; b++)
        ensure(pci[a] != pci[b], "expert-parallel ranks must be on different GPUs");  // kernels wait on each other
    QC_CK(cudaSetDevice(e->device));
    for (uint32_t q = 0; q < W; q++) {
      if (q == R) {
        ep_peer[q] = d_ep;
        continue;
      }
      cudaIpcMemHandle_t h;
      std::memcpy(&h, handles + 64 * q, sizeof h);
      void* ptr = nullptr;
      QC_CK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
      ep_peer[q] = static_cast<uint8_t*>(ptr);
    }
    QC_CK(cudaMemcpy(d_ep_peers, ep_peer, 8 * sizeof(uint8_t*), cudaMemcpyHostToDevice));
    ep_connected = true;
  }
  // Entry check of every call that runs passes.
  void ep_ready() const {
    if (e->ep_world == 1) return;
    ensure(ep_connected, "expert-parallel batch is not connected to its peers");
    ensure(!ep_failed, "an expert-parallel exchange of this batch failed; create a new batch on every rank");
  }

  qc::BatchArgs args() const {
    qc::BatchArgs a{};
    a.tok = d_tok;
    a.kv = d_kv;
    a.kv_floats = kv_floats;
    a.n_layers = e->cfg.layers;
    a.heads = e->cfg.heads;
    a.kvheads = e->cfg.kvheads;
    a.D = e->cfg.head_dim;
    a.ctx = context;
    a.eps = e->cfg.eps;
    a.rope = e->sc.rope;
    return a;
  }

  void create(qc_engine* eng, uint32_t n, uint32_t ctx) {
    e = eng;
    ensure(n > 0 && n <= 4096, "sequence count must be in 1..=4096");
    ensure(ctx > 0 && ctx <= e->context, "batch context must be in 1..=" + std::to_string(e->context));
    n_seqs = n;
    context = ctx;
    pos.assign(n, 0);
    cap = 128;  // tokens per device pass (the MoE tensor-core path is measured up to 128)
    const qc_config& c = e->cfg;
    const uint64_t D = c.head_dim, QD = (uint64_t)c.heads * D, KD = (uint64_t)c.kvheads * D, H = c.hidden, V = c.vocab;
    ensure(D % 32 == 0 && D <= 128 && c.heads / c.kvheads <= 32, "batched attention needs head_dim <= 128 (a multiple of 32) "
           "and at most 32 query heads per KV head");
    QC_CK(cudaSetDevice(e->device));
    kv_floats = (uint64_t)c.kvheads * ctx * D;
    const uint64_t kv_bytes = (uint64_t)n * c.layers * 2 * kv_floats * 4;
    QC_CK(cudaMalloc(&d_kv, kv_bytes));
    QC_CK(cudaMemsetAsync(d_kv, 0, kv_bytes, e->stream));
    for (const qc::LayerDev& L : e->layers) {
      xb_max = std::max(xb_max, qc::xview_bytes(L.q.units, qc::uses_float_x(L.q.kind) || qc::uses_float_x(L.k.kind) ||
                                                               qc::uses_float_x(L.v.kind)));
      xb_max = std::max(xb_max, qc::xview_bytes(L.o.units, qc::uses_float_x(L.o.kind)));
      ensure(qc::batch_matvec_smem(L.q) <= (size_t)kMaxSmem && qc::batch_matvec_smem(L.o) <= (size_t)kMaxSmem,
             "rows too wide for the batched matvec");
    }
    xb_max = std::max(xb_max, qc::xview_bytes(e->out.units, qc::uses_float_x(e->out.kind)));
    ensure(qc::batch_matvec_smem(e->out) <= (size_t)kMaxSmem, "rows too wide for the batched matvec");
    uint64_t o = 0;
    auto take = [&](uint64_t bytes) {
      const uint64_t at = o;
      o = align256(o + bytes);
      return at;
    };
    const uint64_t o_tok = take(cap * sizeof(qc::BatchTok)), o_ids = take(cap * 4), o_osrc = take(cap * 4);
    // tensor-core projections where the formats allow
    auto tc_ok = [&](const qc::MatDesc& m) {
      uint32_t np, ss;
      return !qc::qgemm_shape(m.kind, m.cols, true, &np, &ss);
    };
    tc.assign(4ull * c.layers, 0);
    tc_smin.assign(4ull * c.layers, 1.f);
    uint64_t img_row = 0;
    for (uint32_t l = 0; l < c.layers; l++) {
      const qc::LayerDev& L = e->layers[l];
      const qc::MatDesc* m[4] = {&L.q, &L.k, &L.v, &L.o};
      for (int i = 0; i < 4; i++) {
        if (!tc_ok(*m[i])) continue;
        tc[4 * l + i] = 1;
        img_row = std::max(img_row, qc::qg_image_row_bytes(m[i]->cols, true));
      }
    }
    tc_out = tc_ok(e->out);
    if (tc_out) img_row = std::max(img_row, qc::qg_image_row_bytes(e->out.cols, true));
    const uint64_t o_x = take(cap * H * 4), o_x2 = take(cap * H * 4), o_q = take(cap * QD * 4), o_k = take(cap * KD * 4),
                   o_v = take(cap * KD * 4), o_a = take(cap * QD * 4), o_xv = take((uint64_t)cap * xb_max),
                   o_lg = take(cap * V * 4), o_last = take((uint64_t)n * V * 4), o_flag = take(16),
                   o_rows = take((uint64_t)n * 8), o_sv = take((uint64_t)n * 8),
                   o_img = take((uint64_t)((cap + 15) & ~15u) * img_row), o_hs = take(((cap + 15) & ~15u) * 4);
    QC_CK(cudaMalloc(&d_buf, o));
    QC_CK(cudaMemsetAsync(d_buf, 0, o, e->stream));
    e->ensure_gemm();
    const uint32_t W = e->ep_world;
    e->grow_moe(W * cap);  // (expert parallelism: every rank's tokens of a pass)
    for (uint32_t l = 0; l < c.layers; l++) {  // the tensor-core weight scales of every layer, once
      qc::MoeArgs ma = e->moe_args(l, cap);
      const char* why = qc::moe_tc_supported(ma);
      if (W > 1 && why) throw ApiError(QC_ERR_INVALID, std::string("expert-parallel batches need the tensor-core MoE path: ") + why);
      if (!why) e->moe_scales(l, ma);
    }
    if (W > 1) {
      const uint64_t eb = qc::moe_ep_layout(cap, c.hidden, c.top, W, &ep_set[0], &ep_set[1]);
      QC_CK(cudaMalloc(&d_ep, eb));
      QC_CK(cudaMemsetAsync(d_ep, 0, eb, e->stream));
      QC_CK(cudaMalloc(&d_ep_peers, 8 * sizeof(uint8_t*)));
      for (qc::MoeEp& m : ep_set) {
        m.rank = e->ep_rank;
        m.world = W;
        m.e_n = e->e_n;
        m.peers = d_ep_peers;
        m.own = d_ep;
      }
    }
    QC_CK(cudaMemsetAsync(e->moe_args(0, 1).err, 0, 4, e->stream));
    d_tok = reinterpret_cast<qc::BatchTok*>(d_buf + o_tok);
    d_ids = reinterpret_cast<uint32_t*>(d_buf + o_ids);
    d_osrc = reinterpret_cast<uint32_t*>(d_buf + o_osrc);
    d_x = reinterpret_cast<float*>(d_buf + o_x);
    d_x2 = reinterpret_cast<float*>(d_buf + o_x2);
    d_q = reinterpret_cast<float*>(d_buf + o_q);
    d_k = reinterpret_cast<float*>(d_buf + o_k);
    d_v = reinterpret_cast<float*>(d_buf + o_v);
    d_a = reinterpret_cast<float*>(d_buf + o_a);
    d_xv = d_buf + o_xv;
    d_lg = reinterpret_cast<float*>(d_buf + o_lg);
    d_last = reinterpret_cast<float*>(d_buf + o_last);
    d_flag = reinterpret_cast<uint32_t*>(d_buf + o_flag);
    d_rows = reinterpret_cast<const float**>(d_buf + o_rows);
    d_sv = reinterpret_cast<qc::SamplerDev**>(d_buf + o_sv);
    d_img = d_buf + o_img;
    d_hs = reinterpret_cast<float*>(d_buf + o_hs);
    for (uint32_t l = 0; l < c.layers; l++) {  // Q4_K min-block scales, once
      const qc::LayerDev& L = e->layers[l];
      const qc::MatDesc* m[4] = {&L.q, &L.k, &L.v, &L.o};
      for (int i = 0; i < 4; i++)
        if (tc[4 * l + i]) tc_smin[4 * l + i] = e->dmin_scale(*m[i], 1, d_flag);
    }
    if (tc_out) tc_out_smin = e->dmin_scale(e->out, 1, d_flag);
    QC_CK(cudaStreamSynchronize(e->stream));
  }

  // The activation image of T vectors of K floats (rows src[i] of x, or x's first T rows), RMS-normalized
  // with w when given; their scales go to d_hs.  Q4_K min chunks always (Q6_K GEMMs skip them).
  void tc_image(const float* x, const uint32_t* src, uint32_t T, uint32_t K, const float* w) {
    qc::QgImageArgs ia{};
    ia.x = x;
    ia.xstride = K;
    ia.K = K;
    ia.T = T;
    ia.src = src;
    ia.w = w;
    ia.eps = e->cfg.eps;
    ia.hs_out = d_hs;
    ia.hasmin = 1;
    ia.img = d_img;
    qc::launch_qg_image(ia, (T + 15) & ~15u, e->stream);
  }
  struct TcOut {
    const qc::GemmMat* m;
    float smin;
    float* y;
    const float* add;
    uint64_t ystride;
  };
  // y = W x (+ add) for up to 3 matrices of one format over the current image of T vectors.
  void tc_project(const std::vector<TcOut>& outs, uint32_t T, uint32_t K) {
    if (outs.empty()) return;
    const uint32_t kind = outs[0].m->kind, nimg = (T + 15) & ~15u;
    uint32_t NP = 8, SS = 2;
    qc::qgemm_shape(kind, K, true, &NP, &SS);  // (checked when the batch was created)
    qc::QgArgs q{};
    q.K = K;
    q.NP = NP;
    q.SS = SS;
    q.img_hasmin = 1;
    q.img = d_img;
    q.hs = d_hs;
    q.err = e->moe_args(0, 1).err;
    uint32_t items = 0;
    for (size_t i = 0; i < outs.size(); i++) {
      q.mats[i] = *outs[i].m;
      q.smin[i] = outs[i].smin;
      q.inl[i] = qc::QgGroup{items, T, nimg, 0, (uint32_t)i, 0, outs[i].y, outs[i].add, nullptr, nullptr, outs[i].ystride};
      items += (outs[i].m->rows + 127) / 128 * ((nimg + NP - 1) / NP);
    }
    q.ngroups = (uint32_t)outs.size();
    q.nitems = items;
    qc::launch_qgemm(q, kind, false, std::min<uint32_t>(items, (uint32_t)e->sms), e->stream);
  }

  // One device pass: T tokens (ids in d_ids, sequence and position in d_tok), logits rows for the
  // n_out tokens listed in d_osrc.
  void pass(uint32_t T, uint32_t n_out) {
    const qc_config& c = e->cfg;
    cudaStream_t s = e->stream;
    const uint32_t H = c.hidden, QD = c.heads * c.head_dim, KD = c.kvheads * c.head_dim;
    const qc::BatchArgs ba = args();
    qc::launch_batch_embed(e->embd, d_tok, d_ids, T, H, d_x, s);
    for (uint32_t l = 0; l < c.layers; l++) {
      const qc::LayerDev& L = e->layers[l];
      const uint8_t* t4 = &tc[4 * l];
      // Q, K, V of rms(x) (model.rs:226-240): tensor cores for the formats that allow, else dp4a matvecs
      if (t4[0] || t4[1] || t4[2]) {
        tc_image(d_x, nullptr, T, H, L.attn_norm);
        const qc::MatDesc* m[3] = {&L.q, &L.k, &L.v};
        float* y[3] = {d_q, d_k, d_v};
        const uint64_t st[3] = {QD, KD, KD};
        for (uint32_t kind : {(uint32_t)qc::Q4_K, (uint32_t)qc::Q6_K}) {
          std::vector<TcOut> outs;
          for (int i = 0; i < 3; i++)
            if (t4[i] && m[i]->kind == kind)
              outs.push_back(TcOut{&e->gm(l, i), tc_smin[4 * l + i], y[i], nullptr, st[i]});
          tc_project(outs, T, H);
        }
      }
      if (!(t4[0] && t4[1] && t4[2])) {
        const bool flA = qc::uses_float_x(L.q.kind) || qc::uses_float_x(L.k.kind) || qc::uses_float_x(L.v.kind);
        const uint32_t xbA = qc::xview_bytes(L.q.units, flA);
        qc::launch_batch_stage(d_x, nullptr, T, H, L.q.units, flA, L.attn_norm, c.eps, d_xv, xbA, s);
        if (!t4[0]) qc::launch_batch_matvec(L.q, d_xv, xbA, T, d_q, QD, nullptr, e->sms, s);
        if (!t4[1]) qc::launch_batch_matvec(L.k, d_xv, xbA, T, d_k, KD, nullptr, e->sms, s);
        if (!t4[2]) qc::launch_batch_matvec(L.v, d_xv, xbA, T, d_v, KD, nullptr, e->sms, s);
      }
      qc::launch_batch_qkprep(ba, l, L.q_norm, L.k_norm, d_q, d_k, d_v, T, s);
      qc::launch_batch_attention(ba, l, d_q, d_a, T, s);
      if (t4[3]) {  // x += W_o attn (model.rs:245-248)
        tc_image(d_a, nullptr, T, QD, nullptr);
        tc_project({TcOut{&e->gm(l, 3), tc_smin[4 * l + 3], d_x, d_x, H}}, T, QD);
      } else {
        const uint32_t xbO = qc::xview_bytes(L.o.units, qc::uses_float_x(L.o.kind));
        qc::launch_batch_stage(d_a, nullptr, T, QD, L.o.units, qc::uses_float_x(L.o.kind), nullptr, 0.f, d_xv, xbO, s);
        qc::launch_batch_matvec(L.o, d_xv, xbO, T, d_x, H, d_x, e->sms, s);
      }
      // the MoE half (model.rs:249-287): tensor-core path when the formats allow, else per token
      qc::MoeArgs ma = e->moe_args(l, T);
      if (e->ep_world > 1) {  // tokens of every rank to the experts of this rank, and back
        e->moe_scales(l, ma);
        qc::MoeEp ep = ep_set[ep_layers++ & 1];
        ep.T = T;
        if (const char* why = qc::launch_moe_tc_ep(ma, ep, ep_seq + 1, d_x, d_x2, s)) throw ApiError(QC_ERR_CUDA, why);
        ep_seq += 2;
        std::swap(d_x, d_x2);
      } else if (!qc::moe_tc_supported(ma)) {
        e->moe_scales(l, ma);  // (measured at creation: only reads the cached scales)
        if (const char* why = qc::launch_moe_tc(ma, d_x, d_x2, s)) throw ApiError(QC_ERR_CUDA, why);
        std::swap(d_x, d_x2);
      } else {
        for (uint32_t t = 0; t < T; t++) {
          QC_CK(cudaMemcpyAsync(e->sc.x, d_x + (uint64_t)t * H, H * 4, cudaMemcpyDeviceToDevice, s));
          qc::launch_moe_token(e->dims, e->plan, L, e->sc, e->d_state, s);
          QC_CK(cudaMemcpyAsync(d_x + (uint64_t)t * H, e->sc.x, H * 4, cudaMemcpyDeviceToDevice, s));
        }
      }
      QC_CK(cudaGetLastError());
    }
    if (n_out) {  // model.rs:289-301: output norm, vocabulary rows, finiteness
      if (tc_out) {
        tc_image(d_x, d_osrc, n_out, H, e->out_norm);
        tc_project({TcOut{&e->gemm.back(), tc_out_smin, d_lg, nullptr, c.vocab}}, n_out, H);
      } else {
        const bool flV = qc::uses_float_x(e->out.kind);
        const uint32_t xbV = qc::xview_bytes(e->out.units, flV);
        qc::launch_batch_stage(d_x, d_osrc, n_out, H, e->out.units, flV, e->out_norm, c.eps, d_xv, xbV, s);
        qc::launch_batch_matvec(e->out, d_xv, xbV, n_out, d_lg, c.vocab, nullptr, e->sms, s);
      }
      qc::launch_batch_finite(d_lg, (uint64_t)n_out * c.vocab, d_flag, s);
    }
    QC_CK(cudaGetLastError());
  }

  // Raises the sticky errors of the passes since the last check.
  void check() {
    uint32_t h[2] = {0, 0};
    QC_CK(cudaMemcpyAsync(&h[0], d_flag, 4, cudaMemcpyDeviceToHost, e->stream));
    QC_CK(cudaMemcpyAsync(&h[1], e->moe_args(0, 1).err, 4, cudaMemcpyDeviceToHost, e->stream));
    QC_CK(cudaStreamSynchronize(e->stream));
    QC_CK(cudaMemsetAsync(d_flag, 0, 4, e->stream));
    QC_CK(cudaMemsetAsync(e->moe_args(0, 1).err, 0, 4, e->stream));
    e->check_flags();  // per-token MoE fallback: non-finite router logits
    if (h[1] & 8) {
      ep_failed = true;
      throw ApiError(QC_ERR_CUDA, "expert-parallel exchange: a peer did not reach the barrier within 2 s");
    }
    if (h[1] & 16) {
      ep_failed = true;
      throw ApiError(QC_ERR_INVALID, "expert-parallel ranks ran passes of different token counts");
    }
    if (h[1] & 2) throw ApiError(QC_ERR_CUDA, "tensor-core kernel: a wait timed out");
    if (h[1] & 1) throw ApiError(QC_ERR_NONFINITE, "invalid MoE router");
    if (h[1] & 4) throw ApiError(QC_ERR_NONFINITE, "an expert activation outside the fp16 range of the tensor-core path");
    if (h[0]) throw ApiError(QC_ERR_NONFINITE, "nonfinite model output");
  }

  // Validates a call's sequences and tokens; per token: its position, and whether it is the last
  // token of its sequence in the call (those get logits rows, in call order).
  void plan(const uint32_t* seqs, const uint32_t* toks, uint32_t n, std::vector<qc::BatchTok>& tk,
            std::vector<uint8_t>& last) {
    ensure(n > 0 && seqs, "empty batch");
    std::vector<uint32_t> count(n_seqs, 0);
    for (uint32_t i = 0; i < n; i++) {
      ensure(seqs[i] < n_seqs, "sequence index out of range");
      if (toks) ensure(toks[i] < e->cfg.vocab, "token outside vocabulary", QC_ERR_TOKEN);
      count[seqs[i]]++;
    }
    for (uint32_t q = 0; q < n_seqs; q++)
      ensure((uint64_t)pos[q] + count[q] <= context, "context limit " + std::to_string(context) + " reached",
             QC_ERR_CONTEXT);
    tk.resize(n);
    last.assign(n, 0);
    std::vector<uint32_t> p(pos);
    for (uint32_t i = 0; i < n; i++) tk[i] = qc::BatchTok{seqs[i], p[seqs[i]]++};
    std::vector<uint8_t> seen(n_seqs, 0);
    for (uint32_t i = n; i-- > 0;)
      if (!seen[seqs[i]]) last[i] = seen[seqs[i]] = 1;
  }

  bool started = false;  // a call has changed device state (its sequences are reset if it fails)

  // Forwards of n tokens (ids on the host); logits rows of the last token of each sequence in the
  // call to `logits` (host), in call order.
  void forward(const uint32_t* seqs, const uint32_t* toks, uint32_t n, float* logits) {
    std::vector<qc::BatchTok> tk;
    std::vector<uint8_t> last;
    ensure(toks, "null argument");
    ep_ready();
    plan(seqs, toks, n, tk, last);
    started = true;
    QC_CK(cudaSetDevice(e->device));
    e->grow_moe(cap);
    const uint64_t V = e->cfg.vocab;
    uint32_t rows_done = 0;
    cudaEvent_t t0 = e->ev0, t1 = e->ev1;
    QC_CK(cudaEventRecord(t0, e->stream));
    for (uint32_t b = 0; b < n; b += cap) {
      const uint32_t T = std::min(cap, n - b);
      std::vector<uint32_t> osrc;
      for (uint32_t i = 0; i < T; i++)
        if (last[b + i]) osrc.push_back(i);
      QC_CK(cudaMemcpyAsync(d_tok, tk.data() + b, T * sizeof(qc::BatchTok), cudaMemcpyHostToDevice, e->stream));
      if (toks) QC_CK(cudaMemcpyAsync(d_ids, toks + b, T * 4, cudaMemcpyHostToDevice, e->stream));
      if (!osrc.empty())
        QC_CK(cudaMemcpyAsync(d_osrc, osrc.data(), osrc.size() * 4, cudaMemcpyHostToDevice, e->stream));
      pass(T, (uint32_t)osrc.size());
      for (uint32_t j = 0; j < osrc.size(); j++) {
        const uint32_t sq = tk[b + osrc[j]].seq;
        QC_CK(cudaMemcpyAsync(d_last + sq * V, d_lg + j * V, V * 4, cudaMemcpyDeviceToDevice, e->stream));
        if (logits) QC_CK(cudaMemcpyAsync(logits + (uint64_t)(rows_done + j) * V, d_lg + j * V, V * 4,
                                          cudaMemcpyDeviceToHost, e->stream));
      }
      rows_done += (uint32_t)osrc.size();
      // the ids of the pass were read: synchronize before the next pass overwrites pageable copies
      QC_CK(cudaStreamSynchronize(e->stream));
    }
    QC_CK(cudaEventRecord(t1, e->stream));
    for (uint32_t i = 0; i < n; i++) pos[seqs[i]]++;
    stats.tokens += n;
    check();
    float ms = 0.f;
    QC_CK(cudaEventElapsedTime(&ms, t0, t1));
    stats.matvec_ms += ms;
  }

  // Device arrays for draws of `n` sequences: their latest logits rows and their samplers.
  void stage_draws(qc_sampler* const* smp, const uint32_t* seqs, uint32_t n) {
    std::vector<const float*> rows(n);
    std::vector<qc::SamplerDev*> sv(n);
    bool large = false;
    for (uint32_t i = 0; i < n; i++) {
      ensure(smp[i] && smp[i]->device == e->device, "a sampler lives on another device");
      ensure(seqs[i] < n_seqs, "sequence index out of range");
      ensure(pos[seqs[i]] > 0, "sampling needs the logits of a previous forward");
      rows[i] = d_last + (uint64_t)seqs[i] * e->cfg.vocab;
      sv[i] = smp[i]->d;
      const uint32_t k = smp[i]->top_k;
      large |= (k > 0 && k < e->cfg.vocab ? k : e->cfg.vocab) > qc::sample_exact_max();
    }
    QC_CK(cudaMemcpyAsync(d_rows, rows.data(), n * 8, cudaMemcpyHostToDevice, e->stream));
    QC_CK(cudaMemcpyAsync(d_sv, sv.data(), n * 8, cudaMemcpyHostToDevice, e->stream));
    if (large && !d_sscr) QC_CK(cudaMalloc(&d_sscr, (uint64_t)n_seqs * qc::sample_scratch_bytes(e->cfg.vocab)));
    QC_CK(cudaStreamSynchronize(e->stream));  // the pageable sources above
  }

  void sample(qc_sampler* const* smp, const uint32_t* seqs, uint32_t n, uint32_t* out) {
    ensure(n > 0 && n <= n_seqs && smp && seqs && out, "invalid draws");
    QC_CK(cudaSetDevice(e->device));
    stage_draws(smp, seqs, n);
    QC_CK(qc::launch_sample_batch(d_rows, e->cfg.vocab, n, d_sv, d_ids, d_sscr, e->stream));
    QC_CK(cudaMemcpyAsync(out, d_ids, n * 4, cudaMemcpyDeviceToHost, e->stream));
    QC_CK(cudaStreamSynchronize(e->stream));
    check_samplers(smp, n);
  }

  void check_samplers(qc_sampler* const* smp, uint32_t n) {
    for (uint32_t i = 0; i < n; i++) {
      uint32_t err = 0;
      QC_CK(cudaMemcpy(&err, &smp[i]->d->err, 4, cudaMemcpyDeviceToHost));
      if (err) {
        QC_CK(cudaMemset(&smp[i]->d->err, 0, 4));
        throw ApiError(QC_ERR_INVALID, "invalid logits");
      }
    }
  }

  // The chat loop for n distinct sequences at once: `steps` times, sample every sequence's latest
  // logits with its sampler and run the n sampled ids as one step.  out: steps x n ids (host).
  void decode_sample(qc_sampler* const* smp, const uint32_t* seqs, uint32_t n, uint32_t steps, uint32_t* out) {
    ensure(n > 0 && n <= cap && n <= n_seqs && smp && seqs, "invalid draws");
    ep_ready();
    std::vector<uint8_t> seen(n_seqs, 0);
    for (uint32_t i = 0; i < n; i++) {
      ensure(seqs[i] < n_seqs && !seen[seqs[i]], "sequences of a decode loop must be distinct");
      seen[seqs[i]] = 1;
      ensure((uint64_t)pos[seqs[i]] + steps <= context, "prompt + max-tokens exceed --ctx", QC_ERR_CONTEXT);
    }
    QC_CK(cudaSetDevice(e->device));
    stage_draws(smp, seqs, n);
    started = true;
    if (steps > out_cap) {
      cudaFree(d_out);
      d_out = nullptr;
      out_cap = 0;
      QC_CK(cudaMalloc(&d_out, (uint64_t)steps * n_seqs * 4));
      out_cap = steps;
    }
    const uint64_t V = e->cfg.vocab;
    std::vector<qc::BatchTok> tk(n);
    std::vector<uint32_t> osrc(n);
    for (uint32_t i = 0; i < n; i++) osrc[i] = i;
    QC_CK(cudaMemcpyAsync(d_osrc, osrc.data(), n * 4, cudaMemcpyHostToDevice, e->stream));
    QC_CK(cudaEventRecord(e->ev0, e->stream));
    for (uint32_t st = 0; st < steps; st++) {
      // the ids land in d_ids: the next pass's tokens (d_rows still point at the latest rows)
      QC_CK(qc::launch_sample_batch(d_rows, (uint32_t)V, n, d_sv, d_ids, d_sscr, e->stream));
      QC_CK(cudaMemcpyAsync(d_out + (uint64_t)st * n, d_ids, n * 4, cudaMemcpyDeviceToDevice, e->stream));
      for (uint32_t i = 0; i < n; i++) tk[i] = qc::BatchTok{seqs[i], pos[seqs[i]] + st};
      QC_CK(cudaMemcpyAsync(d_tok, tk.data(), n * sizeof(qc::BatchTok), cudaMemcpyHostToDevice, e->stream));
      pass(n, n);
      for (uint32_t i = 0; i < n; i++)
        QC_CK(cudaMemcpyAsync(d_last + seqs[i] * V, d_lg + i * V, V * 4, cudaMemcpyDeviceToDevice, e->stream));
      QC_CK(cudaStreamSynchronize(e->stream));  // tk is rewritten next step (pageable copy source)
    }
    QC_CK(cudaEventRecord(e->ev1, e->stream));
    for (uint32_t i = 0; i < n; i++) pos[seqs[i]] += steps;
    stats.tokens += (uint64_t)n * steps;
    if (out) QC_CK(cudaMemcpyAsync(out, d_out, (uint64_t)steps * n * 4, cudaMemcpyDeviceToHost, e->stream));
    QC_CK(cudaStreamSynchronize(e->stream));
    check_samplers(smp, n);
    check();
    float ms = 0.f;
    QC_CK(cudaEventElapsedTime(&ms, e->ev0, e->ev1));
    stats.matvec_ms += ms;
  }
};

namespace {

// model.rs:21-90 Config::from_gguf
qc_config config_from(const qc::GgufFile& g) {
  const std::string* arch = g.str("general.architecture");
  ensure(arch && *arch == "qwen3moe", "only qwen3moe architecture is implemented");
  auto get = [&](const char* k) { return g.need_uint(std::string("qwen3moe.") + k); };
  auto opt = [&](const char* k, uint64_t* v) { return g.uint(std::string("qwen3moe.") + k, v); };
  qc_config c{};
  uint64_t v;
  const uint64_t hidden = get("embedding_length"), heads = get("attention.head_count"), top = get("expert_used_count");
  const uint64_t head_dim = opt("attention.key_length", &v) ? v : hidden / (heads ? heads : 1);
  ensure((opt("attention.value_length", &v) ? v : head_dim) == head_dim, "different key/value head sizes unsupported");
  const uint64_t layers = get("block_count"), kvh = get("attention.head_count_kv"), experts = get("expert_count");
  const uint64_t inter =
      opt("expert_feed_forward_length", &v) ? v : get("feed_forward_length") / (top ? top : 1);
  const qc::GgufTensor& te = g.tensor("token_embd.weight");
  ensure(te.dims.size() > 1, "invalid embedding rank");
  const uint64_t maxctx = get("context_length");
  auto u32 = [](uint64_t x) {
    ensure(x <= 0xffffffffull, "invalid Qwen3 MoE config");
    return (uint32_t)x;
  };
  c.hidden = u32(hidden);
  c.heads = u32(heads);
  c.top = u32(top);
  c.head_dim = u32(head_dim);
  c.layers = u32(layers);
  c.kvheads = u32(kvh);
  c.experts = u32(experts);
  c.intermediate = u32(inter);
  c.vocab = u32(te.dims[1]);
  c.max_context = u32(maxctx);
  c.eps = g.real("qwen3moe.attention.layer_norm_rms_epsilon", 1e-6f);
  c.theta = g.real("qwen3moe.rope.freq_base", 1000000.f);
  qc_engine::validate_config(c);
  ensure((opt("rope.dimension_count", &v) ? v : head_dim) == head_dim, "partial rotary dimensions unsupported");
  const std::string* scaling = g.str("qwen3moe.rope.scaling.type");
  ensure(!scaling || *scaling == "none", "RoPE scaling is not implemented; use the original native-context model");
  return c;
}

template <class F>
int api(qc_engine* e, F&& f) {
  try {
    f();
    return QC_OK;
  } catch (const ApiError& x) {
    g_last_error = x.what();
    if (e) e->err = x.what();
    return x.code;
  } catch (const qc::GgufError& x) {
    g_last_error = x.what();
    if (e) e->err = x.what();
    return QC_ERR_INVALID;
  } catch (const std::bad_alloc&) {
    g_last_error = "host allocation failed";
    if (e) e->err = g_last_error;
    return QC_ERR_NOMEM;
  } catch (const std::exception& x) {
    g_last_error = x.what();
    if (e) e->err = x.what();
    return QC_ERR_INVALID;
  }
}

// A forward-type call: on failure the cache and position are reset (model.rs:210-216).
template <class F>
int api_forward(qc_engine* e, F&& f) {
  if (!e) return g_last_error = "null engine", QC_ERR_INVALID;
  const int rc = api(e, f);
  if (rc != QC_OK) e->reset();
  return rc;
}

int create_from(const qc::GgufFile& g, const uint8_t* base, uint32_t context, int device, qc_engine** out,
                uint32_t rank = 0, uint32_t world = 1) {
  std::unique_ptr<qc_engine> e(new qc_engine);
  const qc_config c = config_from(g);
  std::map<std::string, TensorIn> t;
  for (auto& kv : g.tensors) {
    TensorIn ti;
    ti.name = kv.first;
    ti.kind = kv.second.kind;
    ti.dims = kv.second.dims;
    ti.data = base + kv.second.offset;
    ti.len = kv.second.len;
    t[kv.first] = ti;
  }
  e->build(t, c, context, device, rank, world);
  *out = e.release();
  return QC_OK;
}

}  // namespace

#ifdef QC_TRACE
namespace qc {
cudaError_t trace_read(void* host, size_t bytes);
cudaError_t token_trace_read(void* host, size_t bytes);
}
#endif

namespace qc {
// Sets the thread-local message returned by qc_last_error() (used by noalloc.cu).
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace qc

// A failed call that had started on the device resets the sequences it carried.
template <class F>
static int batch_call(qc_batch* b, const uint32_t* seqs, uint32_t n, F&& f) {
  if (!b) return g_last_error = "null batch", QC_ERR_INVALID;
  b->started = false;
  const int rc = api(b->e, f);
  if (rc != QC_OK && b->started && seqs)
    for (uint32_t i = 0; i < n; i++)
      if (seqs[i] < b->n_seqs) b->pos[seqs[i]] = 0;
  return rc;
}

extern "C" {

const char* qc_last_error(void) { return g_last_error.c_str(); }
const char* qc_engine_error(const qc_engine* e) { return e ? e->err.c_str() : g_last_error.c_str(); }

int qc_row_bytes(uint32_t kind, uint64_t cols, uint64_t* out) {
  return api(nullptr, [&] {
    if (const char* e = qc::ggml_row_bytes(kind, cols, out)) throw ApiError(QC_ERR_INVALID, e);
  });
}

int qc_engine_create(const qc_tensor_desc* tensors, size_t n_tensors, const uint8_t* base, size_t base_len,
                     const qc_config* cfg, uint32_t context, int device, qc_engine** out) {
  return api(nullptr, [&] {
    ensure(tensors && cfg && out && (base || !base_len), "null argument");
    *out = nullptr;
    std::map<std::string, TensorIn> t;
    for (size_t k = 0; k < n_tensors; k++) {
      const qc_tensor_desc& d = tensors[k];
      ensure(d.name && d.n_dims >= 1 && d.n_dims <= 3, "invalid tensor descriptor");
      ensure(d.offset <= base_len && d.len <= base_len - d.offset, std::string("truncated tensor ") + d.name);
      TensorIn ti;
      ti.name = d.name;
      ti.kind = d.kind;
      ti.dims.assign(d.dims, d.dims + d.n_dims);
      ti.data = base + d.offset;
      ti.len = d.len;
      ensure(t.emplace(ti.name, ti).second, "duplicate tensor name");
    }
    auto emb = t.find("token_embd.weight");
    ensure(emb != t.end() && emb->second.dims.size() > 1 && emb->second.dims[1] == cfg->vocab,
           "config vocab does not match token_embd.weight");
    std::unique_ptr<qc_engine> e(new qc_engine);
    e->build(t, *cfg, context, device);
    *out = e.release();
  });
}

int qc_engine_create_gguf(const uint8_t* image, size_t len, uint32_t context, int device, qc_engine** out) {
  return api(nullptr, [&] {
    ensure(out && (image || !len), "null argument");
    *out = nullptr;
    qc::GgufFile g;
    g.parse(image, len);
    create_from(g, image, context, device, out);
  });
}

int qc_engine_create_gguf_ep(const uint8_t* image, size_t len, uint32_t context, int device, uint32_t rank,
                             uint32_t world, qc_engine** out) {
  return api(nullptr, [&] {
    ensure(out && (image || !len), "null argument");
    *out = nullptr;
    qc::GgufFile g;
    g.parse(image, len);
    create_from(g, image, context, device, out, rank, world);
  });
}

int qc_engine_ep_handle(qc_engine* e, void* handle, int* device_id) {
  return api(e, [&] {
    ensure(e && handle && device_id, "null argument");
    e->ep_handle(handle, device_id);
  });
}

int qc_engine_ep_connect(qc_engine* e, const void* handles, const int* device_ids) {
  return api(e, [&] {
    ensure(e && handles && device_ids, "null argument");
    e->ep_connect(static_cast<const uint8_t*>(handles), device_ids);
  });
}

int qc_engine_open(const char* path, uint32_t context, int device, qc_engine** out) {
  return api(nullptr, [&] {
    ensure(path && out, "null argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    ensure(fd >= 0, std::string("open ") + path);
    struct stat st;
    fstat(fd, &st);
    const size_t len = (size_t)st.st_size;
    void* map = len ? mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
    close(fd);
    ensure(!len || map != MAP_FAILED, std::string("mmap ") + path);
    struct Unmap {
      void* p;
      size_t n;
      ~Unmap() {
        if (p && p != MAP_FAILED) munmap(p, n);
      }
    } unmap{map, len};
    qc::GgufFile g;
    g.parse(static_cast<const uint8_t*>(map), len);
    create_from(g, static_cast<const uint8_t*>(map), context, device, out);
  });
}

void qc_engine_destroy(qc_engine* e) { delete e; }

int qc_engine_config(const qc_engine* e, qc_config* out) {
  return api(const_cast<qc_engine*>(e), [&] {
    ensure(e && out, "null argument");
    *out = e->cfg;
  });
}

int qc_engine_set_stream(qc_engine* e, void* stream) {
  return api(e, [&] {
    ensure(e, "null engine");
    QC_CK(cudaSetDevice(e->device));
    QC_CK(cudaStreamSynchronize(e->stream));
    e->stream = stream ? static_cast<cudaStream_t>(stream) : e->own;
  });
}

int qc_forward(qc_engine* e, uint32_t token, float* logits) {
  return api_forward(e, [&] { e->forward(token, logits); });
}

int qc_forward_tokens(qc_engine* e, const uint32_t* tokens, size_t n, float* logits) {
  return api_forward(e, [&] {
    ensure(tokens || !n, "null tokens");
    for (size_t i = 0; i < n; i++) e->forward(tokens[i], i + 1 == n ? logits : nullptr);
  });
}

int qc_decode_greedy(qc_engine* e, uint32_t n, uint32_t* tokens_out, float* logits) {
  if (e && (e->pos == 0 || (uint64_t)e->pos + n > e->context))  // argument errors: no reset (main.rs:219-227)
    return api(e, [&] { e->decode(n, tokens_out, logits, true); });
  return api_forward(e, [&] { e->decode(n, tokens_out, logits, true); });
}

int qc_decode_enqueue(qc_engine* e, uint32_t n) {
  if (e && (e->pos == 0 || (uint64_t)e->pos + n > e->context)) return api(e, [&] { e->decode(n, nullptr, nullptr, false); });
  return api_forward(e, [&] { e->decode(n, nullptr, nullptr, false); });
}

// ---- sampling.rs ------------------------------------------------------------------------------
int qc_sampler_create(uint64_t seed, float temperature, uint32_t top_k, float top_p, int device, qc_sampler** out) {
  return api(nullptr, [&] {
    ensure(out, "null argument");
    *out = nullptr;
    ensure(std::isfinite(temperature) && temperature >= 0.f && std::isfinite(top_p) && top_p > 0.f && top_p <= 1.f,
           "invalid sampling parameters");  // sampling.rs:11-19
    std::unique_ptr<qc_sampler> smp(new qc_sampler);
    smp->device = device;
    smp->top_k = top_k;
    QC_CK(cudaSetDevice(device));
    prepare_device(device);
    qc::SamplerDev init{};
    // rand_core 0.6.4 SeedableRng::seed_from_u64: one PCG32 step (XSH-RR output) per 4 key bytes
    uint64_t state = seed;
    for (int i = 0; i < 8; i++) {
      state = state * 6364136223846793005ull + 11634580027462260723ull;
      const uint32_t xs = (uint32_t)(((state >> 18) ^ state) >> 27), rot = (uint32_t)(state >> 59);
      init.key[i] = (xs >> rot) | (xs << ((32 - rot) & 31));
    }
    init.temperature = temperature;
    init.top_k = top_k;
    init.top_p = top_p;
    QC_CK(cudaMalloc(&smp->d, sizeof init));
    QC_CK(cudaMemcpy(smp->d, &init, sizeof init, cudaMemcpyHostToDevice));
    QC_CK(cudaMallocHost(&smp->h, 16));
    QC_CK(cudaStreamCreateWithFlags(&smp->own, cudaStreamNonBlocking));
    *out = smp.release();
  });
}

void qc_sampler_destroy(qc_sampler* s) { delete s; }

int qc_sampler_sample(qc_sampler* s, const float* logits, uint32_t n, void* stream, uint32_t* token) {
  return api(nullptr, [&] {
    ensure(s && token && (logits || !n), "null argument");
    QC_CK(cudaSetDevice(s->device));
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : s->own;
    if (n == 0) throw ApiError(QC_ERR_INVALID, "invalid logits");
    QC_CK(qc::launch_sample(logits, n, s->d, nullptr, s->scratch_for(n), st));
    *token = s->finish(st);
  });
}

int qc_sampler_words(qc_sampler* s, uint32_t n, uint32_t* out) {
  return api(nullptr, [&] {
    ensure(s && (out || !n), "null argument");
    QC_CK(cudaSetDevice(s->device));
    uint32_t* d = nullptr;
    QC_CK(cudaMalloc(&d, (size_t)(n ? n : 1) * 4));
    qc::launch_sampler_words(s->d, n, d, s->own);
    cudaError_t r = cudaGetLastError();
    if (r == cudaSuccess) r = cudaMemcpyAsync(out, d, (size_t)n * 4, cudaMemcpyDeviceToHost, s->own);
    if (r == cudaSuccess) r = cudaStreamSynchronize(s->own);
    cudaFree(d);
    QC_CK(r);
  });
}

int qc_engine_sample(qc_engine* e, qc_sampler* s, uint32_t* token) {
  return api(e, [&] {
    ensure(e && s && token, "null argument");
    ensure(s->device == e->device, "the sampler lives on another device");
    ensure(e->pos > 0, "sampling needs the logits of a previous forward");
    QC_CK(cudaSetDevice(e->device));
    QC_CK(qc::launch_sample(e->sc.logits, e->cfg.vocab, s->d, nullptr, s->scratch_for(e->cfg.vocab), e->stream));
    *token = s->finish(e->stream);
  });
}

int qc_decode_sample(qc_engine* e, qc_sampler* s, uint32_t n, uint32_t* tokens_out, float* logits) {
  if (e && (e->pos == 0 || (uint64_t)e->pos + n > e->context || !s))  // argument errors: no reset
    return api(e, [&] { e->decode_sample(s, n, tokens_out, logits); });
  return api_forward(e, [&] { e->decode_sample(s, n, tokens_out, logits); });
}

int qc_sync(qc_engine* e) {
  return api_forward(e, [&] { e->check_flags(); });
}

int qc_reset(qc_engine* e) {
  return api(e, [&] {
    ensure(e, "null engine");
    e->reset();
  });
}

int qc_position(const qc_engine* e, uint32_t* pos) {
  return api(const_cast<qc_engine*>(e), [&] {
    ensure(e && pos, "null argument");
    *pos = e->pos;
  });
}

int qc_get_stats(const qc_engine* e, qc_stats* out) {
  return api(const_cast<qc_engine*>(e), [&] {
    ensure(e && out, "null argument");
    *out = e->stats;
    out->weight_bytes = e->weight_bytes;
    out->kv_bytes = e->kv_bytes;
  });
}

int qc_engine_set_decode_mode(qc_engine* e, int mode) {
  return api(e, [&] {
    ensure(e, "null engine");
    e->set_mode(mode);
  });
}

int qc_engine_decode_path(const qc_engine* e, int* path, const char** why) {
  return api(const_cast<qc_engine*>(e), [&] {
    ensure(e && path, "null argument");
    *path = e->use_token ? 0 : 1;
    if (why) *why = e->token_why ? e->token_why : "";
  });
}

int qc_moe_layer(qc_engine* e, uint32_t layer, const float* x, uint32_t n_tokens, float* out, int path,
                 float* device_ms) {
  return api(e, [&] {
    ensure(e, "null engine");
    e->moe_layer(layer, x, n_tokens, out, path, device_ms);
  });
}

int qc_profile_step(qc_engine* e, qc_phase_times* out) {
  return api_forward(e, [&] {
    ensure(out != nullptr, "null argument");
    e->profile(out);
  });
}

int qc_logits_device(const qc_engine* e, const float** out) {
  return api(const_cast<qc_engine*>(e), [&] {
    ensure(e && out, "null argument");
    *out = e->sc.logits;
  });
}

int qc_matrix_create(uint32_t kind, uint64_t rows, uint64_t cols, uint64_t experts, const uint8_t* blocks,
                     uint64_t len, int device, qc_matrix** out) {
  return api(nullptr, [&] {
    ensure(out && blocks, "null argument");
    *out = nullptr;
    uint64_t raw_row;
    if (const char* e = qc::ggml_row_bytes(kind, cols, &raw_row)) throw ApiError(QC_ERR_INVALID, e);
    ensure(rows > 0 && experts > 0 && rows <= 0xffffffffull && cols <= 0xffffffffull, "matvec shape mismatch");
    ensure(len == raw_row * rows * experts, "GPU matvec shape mismatch");
    QC_CK(cudaSetDevice(device));
    prepare_device(device);
    std::unique_ptr<qc_matrix> m(new qc_matrix);
    m->device = device;
    const qc::DevLayout lay = qc::dev_layout(kind, cols);
    ensure(lay.group_bytes <= 0xffffffffull, "rows too wide");
    m->bytes = align256(lay.expert_bytes(rows) * experts);
    m->packed = len;
    m->experts = experts;
    QC_CK(cudaMalloc(&m->d, m->bytes));
    QC_CK(cudaMemset(m->d, 0, m->bytes));
    {
      Uploader up(nullptr, raw_row, len);
      up.put(blocks, rows * experts, (uint32_t)rows, raw_row, kind, cols, m->d, lay, lay.expert_bytes(rows));
    }
    QC_CK(cudaDeviceSynchronize());
    m->desc = desc_of(kind, rows, cols, lay, m->d);
    *out = m.release();
  });
}

int qc_matrix_matvec(const qc_matrix* m, uint32_t expert, const float* x, float* y, void* stream) {
  return api(nullptr, [&] {
    ensure(m && x && y, "null argument");
    ensure(expert < m->experts, "expert out of bounds");
    QC_CK(cudaSetDevice(m->device));
    ensure(qc::matvec_smem(m->desc) <= (size_t)kMaxSmem, "row too wide for the shared-memory activation tile");
    qc::launch_matvec(m->desc, expert, x, y, 148, static_cast<cudaStream_t>(stream));
    QC_CK(cudaGetLastError());
  });
}

int qc_matrix_dequant(const qc_matrix* m, uint32_t expert, float* outp, void* stream) {
  return api(nullptr, [&] {
    ensure(m && outp, "null argument");
    ensure(expert < m->experts, "expert out of bounds");
    QC_CK(cudaSetDevice(m->device));
    qc::launch_dequant(m->desc, expert, outp, static_cast<cudaStream_t>(stream));
    QC_CK(cudaGetLastError());
  });
}

int qc_matrix_bytes(const qc_matrix* m, uint64_t* device_bytes, uint64_t* packed_bytes) {
  return api(nullptr, [&] {
    ensure(m, "null argument");
    if (device_bytes) *device_bytes = m->bytes;
    if (packed_bytes) *packed_bytes = m->packed;
  });
}

void qc_matrix_destroy(qc_matrix* m) { delete m; }


// ---- several sequences per step -------------------------------------------------------------
int qc_batch_create(qc_engine* e, uint32_t n_seqs, uint32_t context, qc_batch** out) {
  if (!e) return g_last_error = "null engine", QC_ERR_INVALID;
  return api(e, [&] {
    ensure(out, "null argument");
    *out = nullptr;
    std::unique_ptr<qc_batch> b(new qc_batch);
    b->create(e, n_seqs, context);
    *out = b.release();
  });
}

void qc_batch_destroy(qc_batch* b) { delete b; }

int qc_batch_forward(qc_batch* b, const uint32_t* seq_ids, const uint32_t* tokens, uint32_t n, float* logits) {
  return batch_call(b, seq_ids, n, [&] { b->forward(seq_ids, tokens, n, logits); });
}

int qc_batch_reset(qc_batch* b, uint32_t seq) {
  if (!b) return g_last_error = "null batch", QC_ERR_INVALID;
  return api(b->e, [&] {
    ensure(seq < b->n_seqs || seq == 0xffffffffu, "sequence index out of range");
    for (uint32_t q = 0; q < b->n_seqs; q++)
      if (seq == 0xffffffffu || q == seq) b->pos[q] = 0;
  });
}

int qc_batch_position(const qc_batch* b, uint32_t seq, uint32_t* pos) {
  if (!b) return g_last_error = "null batch", QC_ERR_INVALID;
  return api(b->e, [&] {
    ensure(pos && seq < b->n_seqs, "invalid argument");
    *pos = b->pos[seq];
  });
}

int qc_batch_logits_device(const qc_batch* b, uint32_t seq, const float** out) {
  if (!b) return g_last_error = "null batch", QC_ERR_INVALID;
  return api(b->e, [&] {
    ensure(out && seq < b->n_seqs, "invalid argument");
    *out = b->d_last + (uint64_t)seq * b->e->cfg.vocab;
  });
}

int qc_batch_sample(qc_batch* b, qc_sampler* const* samplers, const uint32_t* seq_ids, uint32_t n, uint32_t* tokens_out) {
  if (!b) return g_last_error = "null batch", QC_ERR_INVALID;
  return api(b->e, [&] { b->sample(samplers, seq_ids, n, tokens_out); });
}

int qc_batch_decode_sample(qc_batch* b, qc_sampler* const* samplers, const uint32_t* seq_ids, uint32_t n, uint32_t steps,
                           uint32_t* tokens_out) {
  return batch_call(b, seq_ids, n, [&] { b->decode_sample(samplers, seq_ids, n, steps, tokens_out); });
}

int qc_batch_ep_handle(qc_batch* b, void* handle, int* device_id) {
  if (!b) return g_last_error = "null batch", QC_ERR_INVALID;
  return api(b->e, [&] {
    ensure(handle && device_id, "null argument");
    b->ep_handle(handle, device_id);
  });
}

int qc_batch_ep_connect(qc_batch* b, const void* handles, const int* device_ids) {
  if (!b) return g_last_error = "null batch", QC_ERR_INVALID;
  return api(b->e, [&] {
    ensure(handles && device_ids, "null argument");
    b->ep_connect(static_cast<const uint8_t*>(handles), device_ids);
  });
}

int qc_batch_stats(const qc_batch* b, qc_stats* out) {
  if (!b) return g_last_error = "null batch", QC_ERR_INVALID;
  return api(b->e, [&] {
    ensure(out, "null argument");
    *out = b->stats;
    out->kv_bytes = (uint64_t)b->n_seqs * b->e->cfg.layers * 2 * b->kv_floats * 4;
    out->weight_bytes = b->e->weight_bytes;
    out->matvecs = ((5ull + 3ull * b->e->cfg.top) * b->e->cfg.layers + 1) * b->stats.tokens;
  });
}

#ifdef QC_TRACE
int qc_trace_read(void* host, size_t bytes) { return qc::trace_read(host, bytes) == cudaSuccess ? 0 : 2; }
int qc_token_trace_read(void* host, size_t bytes) { return qc::token_trace_read(host, bytes) == cudaSuccess ? 0 : 2; }
#endif

int qc_packed_matvec(uint32_t kind, uint64_t rows, uint64_t cols, const uint8_t* blocks, uint64_t len,
                     const float* x, float* y) {
  return api(nullptr, [&] {
    ensure(x && y, "null argument");
    qc_matrix* m = nullptr;
    int rc = qc_matrix_create(kind, rows, cols, 1, blocks, len, 0, &m);
    if (rc) throw ApiError(rc, g_last_error);
    std::unique_ptr<qc_matrix> own(m);
    float *dx = nullptr, *dy = nullptr;
    QC_CK(cudaMalloc(&dx, cols * 4));
    struct Free {
      float** a;
      float** b;
      ~Free() {
        cudaFree(*a);
        cudaFree(*b);
      }
    } fr{&dx, &dy};
    QC_CK(cudaMalloc(&dy, rows * 4));
    QC_CK(cudaMemcpy(dx, x, cols * 4, cudaMemcpyHostToDevice));
    rc = qc_matrix_matvec(m, 0, dx, dy, nullptr);
    if (rc) throw ApiError(rc, g_last_error);
    QC_CK(cudaMemcpy(y, dy, rows * 4, cudaMemcpyDeviceToHost));
  });
}

}  // extern "C"
