// Whole-token persistent decode kernel: one launch runs the entire forward of
// one token (reference model.rs:217-302) on every SM of the GPU.
//
// Grid: one thread block per SM (cooperative launch, so all blocks are
// resident together).  Each block owns a fixed slice of every matrix of every
// layer (row groups of the device layout) and, per layer, runs six phases:
//   P1  rms(x) and the Q/K/V rows of its slice                  (model.rs:228-232)
//   P2  split GQA attention for one (KV head, position range),  (model.rs:233-244, ops.rs:17-98)
//       then the merge of the split softmax states
//   P3  O rows + residual                                       (model.rs:245-248)
//   P4  rms(x') and the router rows                             (model.rs:249-252)
//   P5  top-k + softmax of the router logits, gate/up rows of   (model.rs:253-274, ops.rs:29-56)
//       the selected experts + SwiGLU
//   P6  down rows of all selected experts, weighted combine, residual (model.rs:275-287)
// and then the vocab projection with the greedy argmax (model.rs:289-301).
//
// Blocks exchange activations through per-layer buffers of 8-byte tagged
// values, (token tag << 32) | f32 bits, written and read as single 8-byte
// accesses: a reader polls the values it needs until every one carries the
// current token's tag, so the data is its own ready flag and no separate
// barrier is needed.  Buffers are per layer, so no buffer is rewritten within
// a token, and the tag (DevState::seq) grows by one per token.
//
// Weights move with TMA bulk copies (cp.async.bulk, one thread issues, an
// mbarrier counts the bytes) into two shared-memory regions, issued as soon as
// the region is free and the rows are known: region P holds the block's Q/K/V
// slice, then the gate/up slice of the selected experts, then the next
// layer's Q/K/V slice; region Q holds the O + router slice, then the down
// slice.  Expert weights are issued the moment the block has computed the
// top-k; everything else is in flight one or more phases before it is used.
//
// Every poll gives up after kWaitNs (or as soon as another block has given up)
// and sets DevState::abort, which the host reports as an error; bulk-copy
// waits always run to completion (their copies do not depend on other blocks).
#include <algorithm>

#include "kernels.h"

namespace qc {

namespace {

constexpr int TNT = 512;
constexpr uint32_t kSub = 128;                        // attention positions per online-softmax step
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s

struct Span {
  uint32_t b, e;
  __host__ __device__ uint32_t n() const { return e - b; }
};
// Even split of n items over nb blocks.
__host__ __device__ inline Span span_of(uint32_t n, uint32_t nb, uint32_t c) {
  return {(uint32_t)((uint64_t)n * c / nb), (uint32_t)((uint64_t)n * (c + 1) / nb)};
}
__host__ __device__ inline uint32_t groups_of(uint32_t rows) { return (rows + 7) / 8; }
__host__ __device__ inline uint32_t up16(uint32_t v) { return (v + 15) & ~15u; }

struct TokenParams {
  const LayerDev* layers;  // device array
  MatDesc embd, out;
  const float* out_norm;
  DevState* st;
  float* logits;
  const float2* rope;
  unsigned long long* ll;
  uint64_t ll_layer, ll_qkv, ll_part, ll_attn, ll_xmid, ll_rl, ll_h, ll_xout;
  uint32_t n_layers, hidden, heads, kvheads, D, experts, top, inter, vocab, ctx;
  float eps;
  uint32_t p_bytes, q_bytes, stage_off, misc_off;
  uint32_t smax, out_sg, nsp, nsq;
};

// ---- primitives -----------------------------------------------------------------------------
QC_DEV uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
QC_DEV unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
QC_DEV uint32_t ld_relaxed(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
QC_DEV unsigned long long tagged(float v, uint32_t seq) {
  return ((unsigned long long)seq << 32) | __float_as_uint(v);
}
QC_DEV void ll_put(unsigned long long* p, float v, uint32_t seq) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(tagged(v, seq)) : "memory");
}
QC_DEV void ll_put2(unsigned long long* p, float a, float b, uint32_t seq) {
  asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(tagged(a, seq)), "l"(tagged(b, seq))
               : "memory");
}
QC_DEV void ll_get2(const unsigned long long* p, unsigned long long* a, unsigned long long* b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(*a), "=l"(*b) : "l"(p) : "memory");
}
QC_DEV unsigned long long ll_get(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
QC_DEV bool fresh(unsigned long long v, uint32_t seq) { return (uint32_t)(v >> 32) == seq; }
QC_DEV float val(unsigned long long v) { return __uint_as_float((uint32_t)v); }

// Bounded polling: keep() is false once the wait must end, either because
// another block gave up (abort set) or because kWaitNs passed (then it sets abort).
struct Waiter {
  uint32_t it = 0;
  unsigned long long t0 = 0;
  QC_DEV bool keep(DevState* st, bool watch_abort = true) {
    if ((++it & 31u) != 0) return true;
    const unsigned long long t = gtimer();
    if (t0 == 0) {
      t0 = t;
      return true;
    }
    if (watch_abort && ld_relaxed(&st->abort)) return false;
    if (t - t0 > kWaitNs) {
      atomicOr(&st->abort, 1u);
      return false;
    }
    return true;
  }
};

QC_DEV float ll_wait1(const unsigned long long* p, uint32_t seq, DevState* st) {
  unsigned long long v;
  Waiter w;
  while (!fresh(v = ll_get(p), seq) && w.keep(st)) {
  }
  return val(v);
}

// Tagged values [0, n) of src (16-byte aligned) into dst(i, value); each thread
// polls up to 8 pairs at a time until all carry `seq`.  No barrier inside.
template <class Dst>
QC_DEV void ll_gather(const unsigned long long* src, uint32_t n, Dst dst, uint32_t seq, DevState* st) {
  constexpr int B = 8;
  for (uint32_t base = 0; base < n; base += 2 * B * blockDim.x) {
    unsigned long long a[B], b[B];
    Waiter w;
    bool ok;
    do {
      ok = true;
#pragma unroll
      for (int k = 0; k < B; k++) {
        const uint32_t i = base + 2 * (k * blockDim.x + threadIdx.x);
        a[k] = 0ull;
        b[k] = 0ull;
        if (i < n) {
          ll_get2(src + i, &a[k], &b[k]);
          ok &= fresh(a[k], seq) && (i + 1 >= n || fresh(b[k], seq));
        }
      }
    } while (!ok && w.keep(st));
#pragma unroll
    for (int k = 0; k < B; k++) {
      const uint32_t i = base + 2 * (k * blockDim.x + threadIdx.x);
      if (i < n) dst(i, val(a[k]));
      if (i + 1 < n) dst(i + 1, val(b[k]));
    }
  }
}

// Stage nv tagged vectors of n elements (vector j at src + j*n; n even) as
// consecutive XViews, as stage_vectors does for plain vectors (RMS: nv == 1
// and the vector becomes x * (s * w), ops.rs:3-15).  Ends with __syncthreads().
template <bool RMS>
QC_DEV void stage_ll(uint8_t* mem, uint32_t nv, uint32_t n, uint32_t units, bool with_float,
                     const unsigned long long* __restrict__ src, const float* __restrict__ w, float eps, float* red,
                     uint32_t seq, DevState* st) {
  const uint32_t per = units4(units) * 64;
  const uint32_t total = nv * per, xb = xview_bytes(units, with_float);
  constexpr int P = 2;
  for (uint32_t base = 0; base < total; base += P * blockDim.x * 8) {
    float x[P][8], ww[P][8];
    if constexpr (RMS) {
#pragma unroll
      for (int p = 0; p < P; p++) {
        const uint32_t i0 = base + (p * blockDim.x + threadIdx.x) * 8, e = i0 % per;
#pragma unroll
        for (int k = 0; k < 8; k++) ww[p][k] = i0 < total && e + k < n ? w[e + k] : 0.f;
      }
    }
    Waiter wt;
    bool ok;
    do {
      ok = true;
#pragma unroll
      for (int p = 0; p < P; p++) {
        const uint32_t i0 = base + (p * blockDim.x + threadIdx.x) * 8;
        const uint32_t j = i0 / per, e = i0 % per;
#pragma unroll
        for (int q = 0; q < 4; q++) {
          unsigned long long a = 0ull, b = 0ull;
          if (i0 < total && e + 2 * q < n) {  // n even: the whole pair is inside
            ll_get2(src + (uint64_t)j * n + e + 2 * q, &a, &b);
            ok &= fresh(a, seq) && fresh(b, seq);
          }
          x[p][2 * q] = val(a);
          x[p][2 * q + 1] = val(b);
        }
      }
    } while (!ok && wt.keep(st));
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

// ---- TMA bulk copies and mbarriers ----------------------------------------------------------
QC_DEV void mb_init(uint64_t* b) { asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(b)) : "memory"); }
QC_DEV void mb_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
QC_DEV bool mb_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Copies complete on their own, so this wait ignores the abort flag; only the time limit ends it early.
QC_DEV void mb_wait(uint64_t* b, uint32_t parity, DevState* st) {
  Waiter w;
  while (!mb_try(b, parity) && w.keep(st, false)) {
  }
}
// global -> shared bulk copy; both addresses 16-byte aligned, bytes a multiple of 16.
QC_DEV void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   saddr(dst)),
               "l"(src), "r"(bytes), "r"(saddr(b))
               : "memory");
}
QC_DEV void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
QC_DEV void l2_prefetch(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---- row loops ----------------------------------------------------------------------------------
// Destination of row results: v -> (add ? add[i] + v : v) into ll[i] (tagged) or out[i], i = r - r0.
struct RowsOut {
  const float* add;
  float* out;
  unsigned long long* ll;
  uint32_t seq;
};
template <uint32_t KIND>
__device__ __noinline__ void rows_k(const MatDesc m, uint32_t r0, uint32_t r1, const XView xv, const uint8_t* base,
                                    uint32_t rbase, const RowsOut o, uint32_t warp, uint32_t nw) {
  warp_rows_k<KIND, true>(
      m, r0, r1, xv,
      [&](uint32_t r, const uint8_t** row, const __half** drow) {
        *row = row_ptr(m, base, r - rbase);
        *drow = drow_ptr(m, base, r - rbase);
      },
      [&](uint32_t r, float v) {
        const uint32_t i = r - r0;
        if (o.add) v = __fadd_rn(o.add[i], v);
        if (o.ll) ll_put(o.ll + i, v, o.seq);
        else o.out[i] = v;
      },
      warp, nw);
}
// Rows [r0, r1) of m held in shared memory from row rbase on, by warps (warp, warp + nw, ...) of a subset.
QC_DEV void rows(const MatDesc& m, uint32_t r0, uint32_t r1, const XView& xv, const uint8_t* base, uint32_t rbase,
                 const RowsOut& o, uint32_t warp = threadIdx.x >> 5, uint32_t nw = blockDim.x >> 5) {
  if (r1 <= r0) return;
  switch (m.kind) {
    case Q4_K: rows_k<Q4_K>(m, r0, r1, xv, base, rbase, o, warp, nw); break;
    case Q5_K: rows_k<Q5_K>(m, r0, r1, xv, base, rbase, o, warp, nw); break;
    case Q6_K: rows_k<Q6_K>(m, r0, r1, xv, base, rbase, o, warp, nw); break;
    case Q8_0: rows_k<Q8_0>(m, r0, r1, xv, base, rbase, o, warp, nw); break;
    case Q4_0: rows_k<Q4_0>(m, r0, r1, xv, base, rbase, o, warp, nw); break;
    case F16: rows_k<F16>(m, r0, r1, xv, base, rbase, o, warp, nw); break;
    default: rows_k<F32>(m, r0, r1, xv, base, rbase, o, warp, nw); break;
  }
}

#ifdef QC_TRACE
constexpr uint32_t kTraceLayer = 1;
__device__ unsigned long long g_ttrace[1024][24];
#define QC_TT(k)                                                                                   \
  do {                                                                                             \
    if (threadIdx.x == 0 && blockIdx.x < 1024 && l == kTraceLayer) g_ttrace[blockIdx.x][k] = gtimer(); \
  } while (0)
#define QC_TO(k)                                                                     \
  do {                                                                               \
    if (threadIdx.x == 0 && blockIdx.x < 1024) g_ttrace[blockIdx.x][16 + (k)] = gtimer(); \
  } while (0)
#else
#define QC_TT(k) \
  do {           \
  } while (0)
#define QC_TO(k) \
  do {           \
  } while (0)
#endif

// Shared-memory bytes of the staging and small-array areas (host and device agree on these).
struct AttnSmem {
  uint32_t attn, merge;
};
__host__ __device__ inline AttnSmem attn_stage_bytes(uint32_t G, uint32_t D, uint32_t smax) {
  return {(G * (D + 4) + 2 * D + G * kSub + 3 * G) * 4, (smax * (D + 2) + smax) * 4};
}

// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(TNT, 1) k_token(const __grid_constant__ TokenParams T) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ __align__(8) uint64_t mbar[2 + kMaxTokenSlots];
  __shared__ __align__(16) LayerDev Ld[2];
  __shared__ float red[32];
  __shared__ unsigned long long wbest[TNT / 32];
  __shared__ int wbad[TNT / 32];
  __shared__ int last;

  const uint32_t c = blockIdx.x, nb = gridDim.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = TNT / 32;
  DevState* const st = T.st;
  // written only by the previous launch: final for this one
  const uint32_t seq = st->seq, pos = st->pos, tok_in = st->token;
  const uint32_t token = tok_in < T.vocab ? tok_in : 0;
  if (c == 0 && tid == 0) {  // the token fed at this step (the greedy sequence when steps are chained)
    if (tok_in >= T.vocab) st->bad_token = 1;
    if (st->gen_tokens && st->gen_count < st->gen_cap) st->gen_tokens[st->gen_count] = tok_in;
    st->gen_count = st->gen_count + 1;
  }
  uint8_t* const rP = sm;
  uint8_t* const rQ = sm + T.p_bytes;
  uint8_t* const stg = sm + T.stage_off;
  const uint32_t nslots = T.nsp + T.nsq;
  const uint32_t E = T.experts, top = T.top, D = T.D, G = T.heads / T.kvheads, KP = D + 4;
  const uint32_t QD = T.heads * D, KD = T.kvheads * D;
  // small arrays: [keys E][logits E][sel top][selw top][residual rows][row outputs]
  uint8_t* mp = sm + T.misc_off;
  unsigned long long* const key = reinterpret_cast<unsigned long long*>(mp);
  float* const lg = reinterpret_cast<float*>(mp + up16(E * 8));
  uint32_t* const sel = reinterpret_cast<uint32_t*>(mp + up16(E * 8) + up16(E * 4));
  float* const selw = reinterpret_cast<float*>(mp + up16(E * 8) + up16(E * 4) + up16(top * 4));
  float* const xres = reinterpret_cast<float*>(mp + up16(E * 8) + up16(E * 4) + 2 * up16(top * 4));

  if (tid < sizeof(LayerDev) / 16) cp16(reinterpret_cast<uint8_t*>(&Ld[0]) + 16 * tid,
                                        reinterpret_cast<const uint8_t*>(&T.layers[0]) + 16 * tid);
  cp_commit();
  if (tid == 0) {
    for (uint32_t i = 0; i < 2 + nslots; i++) mb_init(&mbar[i]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  cp_wait_all();
  __syncthreads();
  uint32_t parP = 0, parQ = 0;
  const uint32_t nbl = nb;

  // ---- slices of this block (per layer; byte counts depend on the layer's formats) ----
  struct Slices {
    Span pq, pk, pv, so, sr, sg, sd;
    uint32_t bq, bk, bv, bA, bO, bR, bOR, bGU, bD;
  };
  auto slices = [&](const LayerDev& L) {
    Slices s;
    const uint32_t gq = groups_of(L.q.rows), gk = groups_of(L.k.rows), gv = groups_of(L.v.rows);
    const Span sa = span_of(gq + gk + gv, nbl, c);
    auto part = [&](uint32_t s0, uint32_t n) {
      const uint32_t lo = max(sa.b, s0), hi = min(sa.e, s0 + n);
      return hi > lo ? Span{lo - s0, hi - s0} : Span{0, 0};
    };
    s.pq = part(0, gq);
    s.pk = part(gq, gk);
    s.pv = part(gq + gk, gv);
    s.so = span_of(groups_of(L.o.rows), nbl, c);
    s.sr = span_of(groups_of(L.router.rows), nbl, c);
    s.sg = span_of(top * groups_of(L.gate.rows), nbl, c);
    s.sd = span_of(groups_of(L.down.rows), nbl, c);
    s.bq = s.pq.n() * L.q.group_bytes;
    s.bk = s.pk.n() * L.k.group_bytes;
    s.bv = s.pv.n() * L.v.group_bytes;
    s.bA = s.bq + s.bk + s.bv;
    s.bO = s.so.n() * L.o.group_bytes;
    s.bR = s.sr.n() * L.router.group_bytes;
    s.bOR = s.bO + s.bR;
    s.bGU = s.sg.n() * (L.gate.group_bytes + L.up.group_bytes);
    s.bD = s.sd.n() * top * L.down.group_bytes;
    return s;
  };
  // (thread 0) Q/K/V slice of layer L into region P; O + router slice into region Q
  auto issue_A = [&](const LayerDev& L) {
    const Slices s = slices(L);
    if (!s.bA) return;
    mb_expect(&mbar[0], s.bA);
    if (s.bq) bulk_copy(rP, L.q.w + (uint64_t)s.pq.b * L.q.group_bytes, s.bq, &mbar[0]);
    if (s.bk) bulk_copy(rP + s.bq, L.k.w + (uint64_t)s.pk.b * L.k.group_bytes, s.bk, &mbar[0]);
    if (s.bv) bulk_copy(rP + s.bq + s.bk, L.v.w + (uint64_t)s.pv.b * L.v.group_bytes, s.bv, &mbar[0]);
  };
  auto issue_OR = [&](const LayerDev& L) {
    const Slices s = slices(L);
    if (!s.bOR) return;
    mb_expect(&mbar[1], s.bOR);
    if (s.bO) bulk_copy(rQ, L.o.w + (uint64_t)s.so.b * L.o.group_bytes, s.bO, &mbar[1]);
    if (s.bR) bulk_copy(rQ + s.bO, L.router.w + (uint64_t)s.sr.b * L.router.group_bytes, s.bR, &mbar[1]);
  };
  // vocab projection stages: stage k of this block's groups into slot k % nslots
  const Span sv = span_of(groups_of(T.out.rows), nbl, c);
  const uint32_t osg = T.out_sg, nst = (sv.n() + osg - 1) / osg, slot_bytes = osg * T.out.group_bytes;
  auto slot_ptr = [&](uint32_t j) { return j < T.nsp ? rP + j * slot_bytes : rQ + (j - T.nsp) * slot_bytes; };
  auto issue_stage = [&](uint32_t k) {
    if (k >= nst) return;
    const uint32_t j = k % nslots, g0 = sv.b + k * osg, g1 = min(sv.e, g0 + osg);
    const uint32_t bytes = (g1 - g0) * T.out.group_bytes;
    mb_expect(&mbar[2 + j], bytes);
    bulk_copy(slot_ptr(j), T.out.w + (uint64_t)g0 * T.out.group_bytes, bytes, &mbar[2 + j]);
  };
  if (tid == 0) {
    issue_A(Ld[0]);
    issue_OR(Ld[0]);
  }

  // attention split of this token (the same for every layer)
  const uint32_t time = pos + 1;
  uint32_t S = min(T.smax, (time + kMinChunk - 1) / kMinChunk);
  S = S < 1 ? 1 : S;
  const uint32_t chunk = (time + S - 1) / S;
  S = (time + chunk - 1) / chunk;
  const bool att = c < T.kvheads * S;
  const uint32_t ah = att ? c / S : 0, as = att ? c % S : 0;
  const uint32_t at0 = as * chunk, at1 = min(time, at0 + chunk);
  const float2* const cs = T.rope + (uint64_t)pos * (D / 2);
  const uint8_t* const erow = row_ptr(T.embd, T.embd.w, token);
  const __half* const edrow = drow_ptr(T.embd, T.embd.w, token);

  for (uint32_t l = 0; l < T.n_layers; l++) {
    const LayerDev& L = Ld[l & 1];
    const Slices s = slices(L);
    unsigned long long* const LL = T.ll + (uint64_t)l * T.ll_layer;
    const unsigned long long* const Xin = l ? T.ll + (uint64_t)(l - 1) * T.ll_layer + T.ll_xout : nullptr;
    float* const kc_h = L.kc + (uint64_t)ah * T.ctx * D;
    float* const vc_h = L.vc + (uint64_t)ah * T.ctx * D;
    QC_TT(0);
    // next layer's descriptors into the other slot (last read in layer l-1)
    if (l + 1 < T.n_layers && tid < sizeof(LayerDev) / 16)
      cp16(reinterpret_cast<uint8_t*>(&Ld[(l + 1) & 1]) + 16 * tid,
           reinterpret_cast<const uint8_t*>(&T.layers[l + 1]) + 16 * tid);
    cp_commit();
    if (att && tid == 0) {  // cached K/V rows of this split toward L2
      const uint32_t te = min(at1, pos);
      if (te > at0) {
        const uint32_t bytes = (te - at0) * D * 4;
        for (uint32_t o = 0; o < bytes; o += 16384) {
          l2_prefetch(kc_h + (uint64_t)at0 * D + o / 4, min(16384u, bytes - o));
          l2_prefetch(vc_h + (uint64_t)at0 * D + o / 4, min(16384u, bytes - o));
        }
      }
    }

    // ---- P1: Q, K, V = W rms(x, attn_norm) --------------------------------------------------
    const bool flA = uses_float_x(L.q.kind) || uses_float_x(L.k.kind) || uses_float_x(L.v.kind);
    if (l == 0)
      stage_vectors<true>(
          stg, 1, T.hidden, L.q.units, flA, [&](uint32_t, uint32_t i) { return dequant_one(T.embd, erow, edrow, i); },
          L.attn_norm, T.eps, red);
    else
      stage_ll<true>(stg, 1, T.hidden, L.q.units, flA, Xin, L.attn_norm, T.eps, red, seq, st);
    QC_TT(1);
    const XView xa = xview_at(stg, L.q.units, flA);
    if (s.bA) {
      mb_wait(&mbar[0], parP, st);
      parP ^= 1;
    }
    QC_TT(2);
    if (s.pq.n()) {
      const uint32_t r0 = s.pq.b * 8, r1 = min(L.q.rows, s.pq.e * 8);
      rows(L.q, r0, r1, xa, rP, r0, RowsOut{nullptr, nullptr, LL + T.ll_qkv + r0, seq});
    }
    if (s.pk.n()) {
      const uint32_t r0 = s.pk.b * 8, r1 = min(L.k.rows, s.pk.e * 8);
      rows(L.k, r0, r1, xa, rP + s.bq, r0, RowsOut{nullptr, nullptr, LL + T.ll_qkv + QD + r0, seq});
    }
    if (s.pv.n()) {
      const uint32_t r0 = s.pv.b * 8, r1 = min(L.v.rows, s.pv.e * 8);
      rows(L.v, r0, r1, xa, rP + s.bq + s.bk, r0, RowsOut{nullptr, nullptr, LL + T.ll_qkv + QD + KD + r0, seq});
    }
    __syncthreads();  // staging area reused below
    QC_TT(3);

    // ---- P2: QK-norm, RoPE, KV append, split attention, merge --------------------------------
    if (att) {
      float* const qs = reinterpret_cast<float*>(stg);  // [G][KP] query heads of this KV head
      float* const kn = qs + G * KP;                    // [D] new key (normed, rotated)
      float* const vn = kn + D;                         // [D] new value
      float* const sc = vn + D;                         // [G][kSub] scores, then weights
      float* const mls = sc + G * kSub;                 // [G] running max, [G] running sum, [G] rescale
      const bool has_pos = at1 == time;
      ll_gather(LL + T.ll_qkv + (uint64_t)ah * G * D, G * D,
                [&](uint32_t i, float v) { qs[(i / D) * KP + i % D] = v; }, seq, st);
      if (has_pos) {
        ll_gather(LL + T.ll_qkv + QD + (uint64_t)ah * D, D, [&](uint32_t i, float v) { kn[i] = v; }, seq, st);
        ll_gather(LL + T.ll_qkv + QD + KD + (uint64_t)ah * D, D, [&](uint32_t i, float v) { vn[i] = v; }, seq, st);
      }
      for (uint32_t g = tid; g < G; g += TNT) {
        mls[g] = -INFINITY;
        mls[G + g] = 0.f;
      }
      __syncthreads();
      for (uint32_t g = warp; g < G; g += nw) head_norm_rope(qs + g * KP, L.q_norm, D, T.eps, cs);
      if (has_pos && warp == nw - 1) {  // model.rs:241-243: append k (normed, rotated) and v
        head_norm_rope(kn, L.k_norm, D, T.eps, cs);
        for (uint32_t i = lane; i < D; i += 32) {
          kc_h[(uint64_t)pos * D + i] = kn[i];
          vc_h[(uint64_t)pos * D + i] = vn[i];
        }
      }
      __syncthreads();
      // online softmax over steps of kSub positions; thread (ag, ad4) accumulates 4 dims of head ag
      const float sd = sqrtf((float)D);
      const uint32_t nslot = G * (D / 4), ag = tid / (D / 4), ad4 = tid % (D / 4);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (uint32_t tb = at0; tb < at1; tb += kSub) {
        const uint32_t n = min(kSub, at1 - tb);
        // s[g][t] = (q_g . k_t) / sqrt(D)  (ops.rs:84-91); thread per (t, g), t fastest
        for (uint32_t i = tid; i < n * G; i += TNT) {
          const uint32_t t = i % n, g = i / n;
          const float* kr = tb + t == pos ? kn : kc_h + (uint64_t)(tb + t) * D;
          const float4* k4 = reinterpret_cast<const float4*>(kr);
          const float4* q4 = reinterpret_cast<const float4*>(qs + g * KP);
          float p = 0.f;
          for (uint32_t j = 0; j < D / 4; j++) {
            const float4 a = k4[j], b = q4[j];
            p = fmaf(a.x, b.x, p);
            p = fmaf(a.y, b.y, p);
            p = fmaf(a.z, b.z, p);
            p = fmaf(a.w, b.w, p);
          }
          sc[g * kSub + t] = p / sd;
        }
        __syncthreads();
        for (uint32_t g = warp; g < G; g += nw) {
          float m = -INFINITY;
          for (uint32_t t = lane; t < n; t += 32) m = fmaxf(m, sc[g * kSub + t]);
          m = warp_max(m);
          const float mo = mls[g], mn = fmaxf(mo, m);
          float sum = 0.f;
          for (uint32_t t = lane; t < n; t += 32) {
            const float p = expf(sc[g * kSub + t] - mn);
            sc[g * kSub + t] = p;
            sum += p;
          }
          sum = warp_sum(sum);
          __syncwarp();
          if (lane == 0) {
            const float f = expf(mo - mn);
            mls[2 * G + g] = f;
            mls[G + g] = mls[G + g] * f + sum;
            mls[g] = mn;
          }
        }
        __syncthreads();
        if (tid < nslot) {
          const float f = mls[2 * G + ag];
          acc.x *= f;
          acc.y *= f;
          acc.z *= f;
          acc.w *= f;
          for (uint32_t t = 0; t < n; t++) {
            const float p = sc[ag * kSub + t];
            const float* vr = tb + t == pos ? vn : vc_h + (uint64_t)(tb + t) * D;
            const float4 v = *reinterpret_cast<const float4*>(vr + 4 * ad4);
            acc.x = fmaf(p, v.x, acc.x);
            acc.y = fmaf(p, v.y, acc.y);
            acc.z = fmaf(p, v.z, acc.z);
            acc.w = fmaf(p, v.w, acc.w);
          }
        }
        __syncthreads();
      }
      if (tid < nslot) {
        if (S == 1) {  // one split: normalize and publish the output directly
          const float inv = 1.f / mls[G + ag];
          unsigned long long* o = LL + T.ll_attn + (uint64_t)(ah * G + ag) * D + 4 * ad4;
          ll_put2(o, acc.x * inv, acc.y * inv, seq);
          ll_put2(o + 2, acc.z * inv, acc.w * inv, seq);
        } else {  // partial state [acc[D], m, l] of (head, split)
          unsigned long long* o = LL + T.ll_part + ((uint64_t)(ah * G + ag) * T.smax + as) * (D + 2);
          ll_put2(o + 4 * ad4, acc.x, acc.y, seq);
          ll_put2(o + 4 * ad4 + 2, acc.z, acc.w, seq);
          if (ad4 == 0) ll_put2(o + D, mls[ag], mls[G + ag], seq);
        }
      }
      if (S > 1) {  // this split merges query heads g = as, as + S, ... of its KV head
        float* const pb = reinterpret_cast<float*>(stg);  // [S][D + 2]
        float* const fw = pb + S * (D + 2);               // [S]
        for (uint32_t g = as; g < G; g += S) {
          __syncthreads();
          ll_gather(LL + T.ll_part + (uint64_t)(ah * G + g) * T.smax * (D + 2), S * (D + 2),
                    [&](uint32_t i, float v) { pb[i] = v; }, seq, st);
          __syncthreads();
          if (warp == 0) {
            float M = -INFINITY;
            for (uint32_t k = lane; k < S; k += 32) M = fmaxf(M, pb[k * (D + 2) + D]);
            M = warp_max(M);
            float Lsum = 0.f;
            for (uint32_t k = lane; k < S; k += 32) {
              const float f = expf(pb[k * (D + 2) + D] - M);
              fw[k] = f;
              Lsum = fmaf(pb[k * (D + 2) + D + 1], f, Lsum);
            }
            Lsum = warp_sum(Lsum);
            if (lane == 0) red[0] = 1.f / Lsum;
          }
          __syncthreads();
          for (uint32_t d = tid; d < D; d += TNT) {
            float o = 0.f;
            for (uint32_t k = 0; k < S; k++) o = fmaf(pb[k * (D + 2) + d], fw[k], o);
            ll_put(LL + T.ll_attn + (uint64_t)(ah * G + g) * D + d, o * red[0], seq);
          }
        }
      }
    }
    __syncthreads();
    QC_TT(4);

    // ---- P3: x' = x + W_o attn ----------------------------------------------------------------
    const bool flO = uses_float_x(L.o.kind);
    const uint32_t or0 = s.so.b * 8, or1 = min(L.o.rows, s.so.e * 8);
    for (uint32_t r = or0 + tid; r < or1; r += TNT)
      xres[r - or0] = l == 0 ? dequant_one(T.embd, erow, edrow, r) : ll_wait1(Xin + r, seq, st);
    stage_ll<false>(stg, 1, QD, L.o.units, flO, LL + T.ll_attn, nullptr, 0.f, red, seq, st);
    QC_TT(5);
    if (s.bOR) {
      mb_wait(&mbar[1], parQ, st);
      parQ ^= 1;
    }
    rows(L.o, or0, or1, xview_at(stg, L.o.units, flO), rQ, or0, RowsOut{xres, nullptr, LL + T.ll_xmid + or0, seq});
    __syncthreads();
    QC_TT(6);

    // ---- P4: router logits of rms(x', ffn_norm) (the same vector feeds gate/up) ----------------
    const bool flR = uses_float_x(L.router.kind) || uses_float_x(L.gate.kind) || uses_float_x(L.up.kind);
    stage_ll<true>(stg, 1, T.hidden, L.router.units, flR, LL + T.ll_xmid, L.ffn_norm, T.eps, red, seq, st);
    const XView xf = xview_at(stg, L.router.units, flR);
    QC_TT(7);
    {
      const uint32_t r0 = s.sr.b * 8, r1 = min(L.router.rows, s.sr.e * 8);
      rows(L.router, r0, r1, xf, rQ + s.bO, r0, RowsOut{nullptr, nullptr, LL + T.ll_rl + r0, seq});
    }
    QC_TT(8);

    // ---- P5: top-k with ties to the lower index + softmax over the kept logits, gate/up + SwiGLU
    ll_gather(LL + T.ll_rl, E, [&](uint32_t i, float v) { lg[i] = v; }, seq, st);
    __syncthreads();
    for (uint32_t e = tid; e < E; e += TNT) key[e] = ((unsigned long long)total_key_u(lg[e]) << 32) | (0xffffffffu - e);
    __syncthreads();
    for (uint32_t e = tid; e < E; e += TNT) {
      const unsigned long long ke = key[e];
      uint32_t rank = 0;
      for (uint32_t j = 0; j < E; j++) rank += key[j] > ke;
      if (rank < top) sel[rank] = e;
      if (c == 0 && !isfinite(lg[e])) atomicOr(&st->nonfinite, 1u);
    }
    __syncthreads();
    if (tid == 0) {
      float mx = -INFINITY;  // ops.rs:29-44, in selection order
      for (uint32_t k = 0; k < top; k++) mx = fmaxf(mx, lg[sel[k]]);
      float sum = 0.f;
      for (uint32_t k = 0; k < top; k++) {
        selw[k] = expf(lg[sel[k]] - mx);
        sum = __fadd_rn(sum, selw[k]);
      }
      for (uint32_t k = 0; k < top; k++) selw[k] = selw[k] / sum;
      // the selected experts' gate/up rows into P (Q/K/V consumed in P1), down rows into Q
      proxy_fence();
      const uint32_t gi = groups_of(L.gate.rows);
      if (s.bGU) {
        mb_expect(&mbar[0], s.bGU);
        uint32_t off = 0;
        for (uint32_t i = s.sg.b; i < s.sg.e;) {
          const uint32_t slot = i / gi, g0 = i % gi, ng = min(gi - g0, s.sg.e - i), e = sel[slot];
          bulk_copy(rP + off, L.gate.w + (uint64_t)e * L.gate.expert_stride + (uint64_t)g0 * L.gate.group_bytes,
                    ng * L.gate.group_bytes, &mbar[0]);
          off += ng * L.gate.group_bytes;
          bulk_copy(rP + off, L.up.w + (uint64_t)e * L.up.expert_stride + (uint64_t)g0 * L.up.group_bytes,
                    ng * L.up.group_bytes, &mbar[0]);
          off += ng * L.up.group_bytes;
          i += ng;
        }
      }
      if (s.bD) {
        mb_expect(&mbar[1], s.bD);
        const uint32_t per = s.sd.n() * L.down.group_bytes;
        for (uint32_t k = 0; k < top; k++)
          bulk_copy(rQ + k * per,
                    L.down.w + (uint64_t)sel[k] * L.down.expert_stride + (uint64_t)s.sd.b * L.down.group_bytes, per,
                    &mbar[1]);
      }
    }
    __syncthreads();
    QC_TT(9);
    const uint32_t gi = groups_of(L.gate.rows), nitem = s.sg.n();
    float* const gout = xres;  // [2][nitem * 8] gate then up results
    if (s.bGU) {
      mb_wait(&mbar[0], parP, st);
      parP ^= 1;
    }
    QC_TT(10);
    {
      uint32_t off = 0;
      for (uint32_t i = s.sg.b; i < s.sg.e;) {
        const uint32_t g0 = i % gi, ng = min(gi - g0, s.sg.e - i), it0 = i - s.sg.b;
        const uint32_t r0 = g0 * 8, r1 = min(L.gate.rows, (g0 + ng) * 8);
        rows(L.gate, r0, r1, xf, rP + off, r0, RowsOut{nullptr, gout + it0 * 8, nullptr, 0});
        off += ng * L.gate.group_bytes;
        rows(L.up, r0, r1, xf, rP + off, r0, RowsOut{nullptr, gout + (nitem + it0) * 8, nullptr, 0});
        off += ng * L.up.group_bytes;
        i += ng;
      }
    }
    __syncthreads();
    for (uint32_t idx = tid; idx < nitem * 8; idx += TNT) {
      const uint32_t i = s.sg.b + idx / 8, slot = i / gi, r = (i % gi) * 8 + idx % 8;
      if (r < T.inter) {
        const float gv = gout[idx], uv = gout[nitem * 8 + idx];
        ll_put(LL + T.ll_h + (uint64_t)slot * T.inter + r, __fmul_rn(gv / (1.f + expf(-gv)), uv), seq);
      }
    }
    cp_wait_all();  // the next layer's descriptors
    __syncthreads();
    if (tid == 0) {  // region P is free: next layer's Q/K/V slice, or the first vocab stages
      proxy_fence();
      if (l + 1 < T.n_layers) issue_A(Ld[(l + 1) & 1]);
      else
        for (uint32_t k = 0; k < T.nsp; k++) issue_stage(k);
    }
    QC_TT(11);

    // ---- P6: x'' = x' + sum_s w_s W_down[e_s] h_s, in selection order --------------------------
    const bool flD = uses_float_x(L.down.kind);
    const uint32_t dr0 = s.sd.b * 8, dr1 = min(L.down.rows, s.sd.e * 8), nd = s.sd.n() * 8;
    float* const dres = xres;           // [nd] x' rows of this block
    float* const dout = xres + nd;      // [top][nd]
    for (uint32_t r = dr0 + tid; r < dr1; r += TNT) dres[r - dr0] = ll_wait1(LL + T.ll_xmid + r, seq, st);
    stage_ll<false>(stg, top, T.inter, L.down.units, flD, LL + T.ll_h, nullptr, 0.f, red, seq, st);
    QC_TT(12);
    const uint32_t xb = xview_bytes(L.down.units, flD);
    if (s.bD) {
      mb_wait(&mbar[1], parQ, st);
      parQ ^= 1;
    }
    QC_TT(13);
    if (dr1 > dr0) {
      const uint32_t per = nw >= top ? nw / top : 1, pbytes = s.sd.n() * L.down.group_bytes;
      for (uint32_t k = warp / per; k < top; k += nw / per)
        rows(L.down, dr0, dr1, xview_at(stg + k * xb, L.down.units, flD), rQ + k * pbytes, dr0,
             RowsOut{nullptr, dout + k * nd, nullptr, 0}, warp % per, per);
    }
    __syncthreads();
    for (uint32_t r = dr0 + tid; r < dr1; r += TNT) {
      float acc = 0.f;
      for (uint32_t k = 0; k < top; k++) acc = __fadd_rn(acc, __fmul_rn(selw[k], dout[k * nd + r - dr0]));
      ll_put(LL + T.ll_xout + r, __fadd_rn(dres[r - dr0], acc), seq);
    }
    __syncthreads();
    if (tid == 0) {  // region Q is free: next layer's O + router slice, or the remaining vocab stages
      proxy_fence();
      if (l + 1 < T.n_layers) issue_OR(Ld[(l + 1) & 1]);
      else
        for (uint32_t k = T.nsp; k < nslots; k++) issue_stage(k);
    }
    QC_TT(14);
  }

  // ---- logits = W_out rms(x, output_norm); finiteness; greedy argmax (ties to the lower index) --
  const MatDesc& mo = T.out;
  const bool flV = uses_float_x(mo.kind);
  stage_ll<true>(stg, 1, T.hidden, mo.units, flV, T.ll + (uint64_t)(T.n_layers - 1) * T.ll_layer + T.ll_xout,
                 T.out_norm, T.eps, red, seq, st);
  QC_TO(0);
  const XView xv = xview_at(stg, mo.units, flV);
  unsigned long long best = 0ull;
  bool bad = false;
  for (uint32_t k = 0; k < nst; k++) {
    const uint32_t j = k % nslots;
    mb_wait(&mbar[2 + j], (k / nslots) & 1, st);
    const uint32_t g0 = sv.b + k * osg, g1 = min(sv.e, g0 + osg);
    const uint32_t r0 = g0 * 8, r1 = min(mo.rows, g1 * 8);
    warp_rows<true>(mo, r0, r1, xv, SmemRows{&mo, slot_ptr(j), r0}, [&](uint32_t r, float p) {
      T.logits[r] = p;
      bad |= !isfinite(p);
      const unsigned long long kk = ((unsigned long long)total_key_u(p) << 32) | (0xffffffffu - r);
      best = kk > best ? kk : best;
    });
    __syncthreads();
    if (tid == 0) {
      proxy_fence();
      issue_stage(k + nslots);
    }
  }
  QC_TO(1);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  const int anybad = __any_sync(0xffffffffu, bad);
  if (lane == 0) {
    wbest[warp] = best;
    wbad[warp] = anybad;
  }
  __syncthreads();
  if (tid == 0) {
    unsigned long long b = 0ull;
    int bb = 0;
    for (uint32_t w = 0; w < nw; w++) {
      b = wbest[w] > b ? wbest[w] : b;
      bb |= wbad[w];
    }
    if (bb) atomicOr(&st->nonfinite, 2u);
    if (b) atomicMax(&st->best, b);
    __threadfence();
    last = atomicAdd(&st->output_done, 1u) == nb - 1;
  }
  __syncthreads();
  if (!last || tid != 0) return;
  __threadfence();  // every block's argmax is in
  const unsigned long long b = atomicAdd(&st->best, 0ull);
  st->token = 0xffffffffu - (uint32_t)(b & 0xffffffffu);
  st->pos = pos + 1;
  st->seq = seq + 1;
  st->best = 0ull;
  st->output_done = 0;
  QC_TO(2);
}

}  // namespace

// ---------------------------------------------------------------------------------------------
// Host side.

static uint32_t g_token_smem_cap = 0;  // dynamic shared memory the kernel may use (set by token_prepare)

cudaError_t token_prepare(int max_smem) {
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, k_token);
  if (e != cudaSuccess) return e;
  int dev = 0, optin = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return e;
  int cap = optin - (int)fa.sharedSizeBytes;
  if (max_smem > 0 && cap > max_smem) cap = max_smem;
  if (cap < 0) cap = 0;
  e = cudaFuncSetAttribute(k_token, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
  if (e == cudaSuccess) g_token_smem_cap = (uint32_t)cap;
  return e;
}

const char* plan_token(const StepArgs& a, int max_smem, TokenPlan* p) {
  const DecodeDims& d = a.dims;
  const uint32_t nb = (uint32_t)a.sms, G = d.heads / d.kvheads, D = d.head_dim;
  if (nb < d.kvheads || nb == 0) return "fewer SMs than KV heads";
  if (G * (D / 4) > (uint32_t)TNT) return "query heads per KV head x head_dim / 4 exceeds the block size";
  if (d.hidden % 2 || (d.heads * D) % 2 || d.inter % 2) return "hidden, heads*head_dim and the expert width must be even";
  TokenPlan t{};
  t.nb = nb;
  t.smax = std::max(1u, std::min(nb / d.kvheads, (d.ctx + kMinChunk - 1) / kMinChunk));
  const uint32_t cap = std::min<uint32_t>(g_token_smem_cap, (uint32_t)max_smem);
  uint32_t P = 0, Q = 0, stage = 0, res = 0, outs = 0;
  const AttnSmem as = attn_stage_bytes(G, D, t.smax);
  stage = std::max(as.attn, as.merge);
  for (uint32_t l = 0; l < a.n_layers; l++) {
    const LayerDev& L = a.layers[l];
    if (L.q.units != L.k.units || L.q.units != L.v.units || L.q.lpr != L.k.lpr || L.q.lpr != L.v.lpr ||
        L.router.units != L.gate.units || L.gate.units != L.up.units || L.gate.lpr != L.up.lpr ||
        L.gate.rows != d.inter || L.down.cols != d.inter || L.down.rows != d.hidden || L.o.rows != d.hidden)
      return "unexpected matrix shapes";
    const bool flA = uses_float_x(L.q.kind) || uses_float_x(L.k.kind) || uses_float_x(L.v.kind);
    const bool flR = uses_float_x(L.router.kind) || uses_float_x(L.gate.kind) || uses_float_x(L.up.kind);
    stage = std::max(stage, xview_bytes(L.q.units, flA));
    stage = std::max(stage, xview_bytes(L.o.units, uses_float_x(L.o.kind)));
    stage = std::max(stage, xview_bytes(L.router.units, flR));
    stage = std::max(stage, d.top * xview_bytes(L.down.units, uses_float_x(L.down.kind)));
    const uint32_t gq = groups_of(L.q.rows), gk = groups_of(L.k.rows), gv = groups_of(L.v.rows);
    for (uint32_t c = 0; c < nb; c++) {
      const Span sa = span_of(gq + gk + gv, nb, c);
      uint32_t bA = 0;
      const uint32_t seg0[3] = {0, gq, gq + gk}, segn[3] = {gq, gk, gv}, gb[3] = {L.q.group_bytes, L.k.group_bytes, L.v.group_bytes};
      for (int k = 0; k < 3; k++) {
        const uint32_t lo = std::max(sa.b, seg0[k]), hi = std::min(sa.e, seg0[k] + segn[k]);
        if (hi > lo) bA += (hi - lo) * gb[k];
      }
      const Span so = span_of(groups_of(L.o.rows), nb, c), sr = span_of(groups_of(L.router.rows), nb, c);
      const Span sg = span_of(d.top * groups_of(L.gate.rows), nb, c), sd = span_of(groups_of(L.down.rows), nb, c);
      const uint32_t bOR = so.n() * L.o.group_bytes + sr.n() * L.router.group_bytes;
      const uint32_t bGU = sg.n() * (L.gate.group_bytes + L.up.group_bytes);
      const uint32_t bD = sd.n() * d.top * L.down.group_bytes;
      P = std::max(P, std::max(bA, bGU));
      Q = std::max(Q, std::max(bOR, bD));
      res = std::max(res, std::max(so.n() * 8, sd.n() * 8));
      outs = std::max(outs, std::max(2 * sg.n() * 8, (d.top + 1) * sd.n() * 8));
    }
  }
  stage = std::max(stage, xview_bytes(a.out.units, uses_float_x(a.out.kind)));
  // vocab stages: about 40 KB each, at least two slots over P and Q
  const uint32_t ogb = a.out.group_bytes;
  const uint32_t vper = (groups_of(a.out.rows) + nb - 1) / nb;
  uint32_t sg = std::max(1u, std::min(40960u / ogb, (vper + 1) / 2));
  const uint32_t slot = sg * ogb;
  P = std::max(P, slot);
  Q = std::max(Q, slot);
  P = up16(P);
  Q = up16(Q);
  t.out_sg = sg;
  t.nsp = std::min(P / slot, kMaxTokenSlots / 2);
  t.nsq = std::min(Q / slot, kMaxTokenSlots - t.nsp);
  t.p_bytes = P;
  t.q_bytes = Q;
  t.stage_off = P + Q;
  t.misc_off = t.stage_off + up16(stage);
  const uint32_t misc = up16(d.experts * 8) + up16(d.experts * 4) + 2 * up16(d.top * 4) + up16(std::max(res, outs) * 4);
  t.smem = t.misc_off + misc;
  if (t.smem > cap) return "the per-block weight slices and staging exceed the shared memory of one SM";
  // exchange buffers (8-byte tagged values), each a multiple of 2 values
  auto ev = [](uint64_t n) { return (n + 1) & ~1ull; };
  const uint64_t QD = (uint64_t)d.heads * D, KD = (uint64_t)d.kvheads * D;
  uint64_t o = 0;
  t.ll_qkv = o;
  o += ev(QD + 2 * KD);
  t.ll_part = o;
  o += ev((uint64_t)d.heads * t.smax * (D + 2));
  t.ll_attn = o;
  o += ev(QD);
  t.ll_xmid = o;
  o += ev(d.hidden);
  t.ll_rl = o;
  o += ev(d.experts);
  t.ll_h = o;
  o += ev((uint64_t)d.top * d.inter);
  t.ll_xout = o;
  o += ev(d.hidden);
  t.ll_layer = o;
  *p = t;
  return nullptr;
}

void launch_token(const StepArgs& a, const TokenPlan& p, unsigned long long* ll, bool cooperative, cudaStream_t s) {
  TokenParams T{};
  T.layers = a.layers_dev;
  T.embd = a.embd;
  T.out = a.out;
  T.out_norm = a.out_norm;
  T.st = a.st;
  T.logits = a.sc.logits;
  T.rope = a.sc.rope;
  T.ll = ll;
  T.ll_layer = p.ll_layer;
  T.ll_qkv = p.ll_qkv;
  T.ll_part = p.ll_part;
  T.ll_attn = p.ll_attn;
  T.ll_xmid = p.ll_xmid;
  T.ll_rl = p.ll_rl;
  T.ll_h = p.ll_h;
  T.ll_xout = p.ll_xout;
  const DecodeDims& d = a.dims;
  T.n_layers = a.n_layers;
  T.hidden = d.hidden;
  T.heads = d.heads;
  T.kvheads = d.kvheads;
  T.D = d.head_dim;
  T.experts = d.experts;
  T.top = d.top;
  T.inter = d.inter;
  T.vocab = d.vocab;
  T.ctx = d.ctx;
  T.eps = d.eps;
  T.p_bytes = p.p_bytes;
  T.q_bytes = p.q_bytes;
  T.stage_off = p.stage_off;
  T.misc_off = p.misc_off;
  T.smax = p.smax;
  T.out_sg = p.out_sg;
  T.nsp = p.nsp;
  T.nsq = p.nsq;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nb);
  cfg.blockDim = dim3(TNT);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cooperative ? 1 : 0;
  cudaLaunchKernelEx(&cfg, k_token, T);
}

#ifdef QC_TRACE
cudaError_t token_trace_read(void* host, size_t bytes) { return cudaMemcpyFromSymbol(host, g_ttrace, bytes); }
#endif

}  // namespace qc
