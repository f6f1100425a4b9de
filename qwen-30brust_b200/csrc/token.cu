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
constexpr uint32_t kTokMinChunk = 32;  // attention positions per split of the whole-token kernel, at least
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
  uint32_t smax, out_sg, nsp, nsq, nsegs, part_floats;
  // expert parallelism: rank of world, local experts [e_lo, e_lo + e_n), ranks' exchange buffers
  uint32_t world, rank, e_lo, e_n;
  unsigned long long* const* peers;
  uint64_t ll_moe;
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
// System-scope forms for the expert-parallel exchange: written by a peer GPU over NVLink.
QC_DEV void ll_put_sys(unsigned long long* p, float v, uint32_t seq) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(tagged(v, seq)) : "memory");
}
QC_DEV void ll_get2_sys(const unsigned long long* p, unsigned long long* a, unsigned long long* b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(*a), "=l"(*b) : "l"(p) : "memory");
}
QC_DEV unsigned long long ll_get_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
QC_DEV bool fresh(unsigned long long v, uint32_t seq) { return (uint32_t)(v >> 32) == seq; }
QC_DEV float val(unsigned long long v) { return __uint_as_float((uint32_t)v); }

// Phase timestamps of thread 0 of each block (diagnostic builds only): slots 0-15
// and 20-47 for one layer, 16-19 for the vocab projection.
#ifdef QC_TRACE
__device__ unsigned long long g_ttrace[1024][48];
QC_DEV void trace_at(bool on, int k) {
  if (on && threadIdx.x == 0 && blockIdx.x < 1024) g_ttrace[blockIdx.x][k] = gtimer();
}
#else
QC_DEV void trace_at(bool, int) {}
#endif
#define QC_TT(k) trace_at(l == 1, k)
#define QC_TO(k) trace_at(true, 16 + (k))

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

// As ll_wait1 for a value that a peer GPU writes.
QC_DEV float ll_wait1_sys(const unsigned long long* p, uint32_t seq, DevState* st) {
  unsigned long long v;
  Waiter w;
  while (!fresh(v = ll_get_sys(p), seq) && w.keep(st)) {
  }
  return val(v);
}

// Tagged values [0, n) of src (16-byte aligned) into dst(i, value); each thread
// polls up to 2 pairs at a time until all carry `seq`.  No barrier inside.  (Small unroll
// factors here and in stage_ll keep the kernel's code path per layer short: instruction fetch
// is its largest stall, and B = 2 / P = 1 measured 6% faster than B = 8 / P = 2.)
template <class Dst>
QC_DEV void ll_gather(const unsigned long long* src, uint32_t n, Dst dst, uint32_t seq, DevState* st) {
  constexpr int B = 2;
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
                     uint32_t seq, DevState* st, bool trace = false, int tslot = 0,
                     const unsigned long long* add = nullptr, uint32_t nadd = 0) {
  // (with nadd > 0, nv == 1 and each element is src[i] + add[0*n + i] + add[1*n + i] + ..., the adds
  // written by peer GPUs and read at system scope, summed in order)
  const uint32_t per = units4(units) * 64;
  const uint32_t total = nv * per, xb = xview_bytes(units, with_float);
  constexpr int P = 1;
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
        if (nadd && i0 < total)  // (expert parallelism) the peers' vectors, added in order
          for (uint32_t q = 0; q < 8 && e + q < n; q += 2)
            for (uint32_t k = 0; k < nadd; k++) {
              unsigned long long a, b;
              ll_get2_sys(add + (uint64_t)k * n + e + q, &a, &b);
              ok &= fresh(a, seq) && fresh(b, seq);
              x[p][q] = __fadd_rn(x[p][q], val(a));
              x[p][q + 1] = __fadd_rn(x[p][q + 1], val(b));
            }
      }
    } while (!ok && wt.keep(st));
    trace_at(trace, tslot);
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
  bytes &= ~15u;
  if (bytes) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
// A layer's norm vectors toward L2 (they are read element-wise by every block).
QC_DEV void prefetch_vectors(const LayerDev& L, uint32_t hidden, uint32_t D) {
  l2_prefetch(L.attn_norm, hidden * 4);
  l2_prefetch(L.ffn_norm, hidden * 4);
  l2_prefetch(L.q_norm, D * 4);
  l2_prefetch(L.k_norm, D * 4);
}

// ---- row loops ----------------------------------------------------------------------------------
// A run of rows of one matrix held in shared memory: rows [r0, r1), row rbase at `base`.  Each
// result v (plus add[i], i = r - r0) goes to ll[i] as a tagged value, or to out[i].
struct Seg {
  const uint8_t* base;
  const float* add;
  float* out;
  unsigned long long* ll;
  uint32_t r0, r1, rbase;
  uint32_t main_bytes, d_bytes, group_bytes, kind;
};
__host__ __device__ inline Seg make_seg(const MatDesc& m, const uint8_t* base, uint32_t r0, uint32_t r1,
                                        uint32_t rbase, const float* add, float* out, unsigned long long* ll) {
  return Seg{base, add, out, ll, r0, r1, rbase, m.main_bytes, m.d_bytes, m.group_bytes, m.kind};
}
QC_DEV const uint8_t* seg_row(const Seg* q, uint32_t r) {
  const uint32_t rr = r - q->rbase;
  return q->base + (rr >> 3) * q->group_bytes + (rr & 7) * q->main_bytes;
}
QC_DEV const __half* seg_drow(const Seg* q, uint32_t r) {
  const uint32_t rr = r - q->rbase;
  return reinterpret_cast<const __half*>(q->base + (rr >> 3) * q->group_bytes + 8 * q->main_bytes + (rr & 7) * q->d_bytes);
}
QC_DEV void seg_emit(const Seg* q, uint32_t r, float v, uint32_t seq) {
  const uint32_t i = r - q->r0;
  if (q->add) v = __fadd_rn(q->add[i], v);
  if (q->ll) ll_put(q->ll + i, v, seq);
  else q->out[i] = v;
}

// Rows of the runs sg[0..nseg) (one format; activation XView of `units` units), joint row index ri
// in [0, R), R = total rows.  Warps split each row's units: a group of 8 lanes covers 8
// consecutive units of one row, 4 rows per warp step, so a warp reads only its own 8 units of the
// activation (once, broadcast to its 4 row slots) and every unit of the weights once.  The sum of
// a row over unit group ug goes to part[ug * R + ri]; rows_finish adds the groups in order.
QC_DEV uint32_t unit_groups(uint32_t units) { return (units + 7) / 8; }
// (part[ug * Rtot + roff + ri] when these runs are a part of a larger table.)
template <uint32_t KIND>
__device__ __noinline__ void rows_us(const Seg* sg, uint32_t nseg, uint32_t units, const XView xv, float* part,
                                     uint32_t Rtot, uint32_t roff, uint32_t warp, uint32_t nw) {
  uint32_t R = 0;
  for (uint32_t k = 0; k < nseg; k++) R += sg[k].r1 - sg[k].r0;
  const uint32_t UG = unit_groups(units), lane = threadIdx.x & 31, rg = lane >> 3, j = lane & 7;
  const uint32_t wpg = UG <= nw ? nw / UG : 1;
  for (uint32_t ug = warp / wpg; ug < UG && warp < wpg * (UG <= nw ? UG : nw); ug += (UG <= nw ? UG : nw)) {
    const uint32_t u = ug * 8 + j;
    const bool uon = u < units;
    const auto ux = load_x<KIND>(xv, uon ? u : 0);
    uint32_t s = 0, first = 0;  // segment of ri; ri only grows
    for (uint32_t rb = (warp % wpg) * 4; rb < R; rb += 4 * wpg) {  // the same trip count for the whole warp
      const uint32_t ri = rb + rg;
      float v = 0.f;
      if (ri < R) {
        while (ri >= first + sg[s].r1 - sg[s].r0) {
          first += sg[s].r1 - sg[s].r0;
          s++;
        }
        const Seg* q = sg + s;
        const uint32_t r = q->r0 + ri - first;
        if (uon) v = unit_dot<KIND, true>(seg_row(q, r), seg_drow(q, r), u, ux);
      }
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      if (j == 0 && ri < R) part[ug * Rtot + roff + ri] = v;
    }
  }
}
// All runs of a table (consecutive runs of one format go to one call); no barrier inside.
QC_DEV void run_rows(const Seg* sg, uint32_t nseg, uint32_t units, const XView& xv, float* part,
                     uint32_t warp = threadIdx.x >> 5, uint32_t nw = blockDim.x >> 5) {
  uint32_t Rtot = 0;
  for (uint32_t k = 0; k < nseg; k++) Rtot += sg[k].r1 - sg[k].r0;
  uint32_t roff = 0;
  for (uint32_t i = 0; i < nseg;) {
    uint32_t j = i + 1, R = sg[i].r1 - sg[i].r0;
    while (j < nseg && sg[j].kind == sg[i].kind) R += sg[j].r1 - sg[j].r0, j++;
    switch (sg[i].kind) {
      case Q4_K: rows_us<Q4_K>(sg + i, j - i, units, xv, part, Rtot, roff, warp, nw); break;
      case Q5_K: rows_us<Q5_K>(sg + i, j - i, units, xv, part, Rtot, roff, warp, nw); break;
      case Q6_K: rows_us<Q6_K>(sg + i, j - i, units, xv, part, Rtot, roff, warp, nw); break;
      case Q8_0: rows_us<Q8_0>(sg + i, j - i, units, xv, part, Rtot, roff, warp, nw); break;
      case Q4_0: rows_us<Q4_0>(sg + i, j - i, units, xv, part, Rtot, roff, warp, nw); break;
      case F16: rows_us<F16>(sg + i, j - i, units, xv, part, Rtot, roff, warp, nw); break;
      default: rows_us<F32>(sg + i, j - i, units, xv, part, Rtot, roff, warp, nw); break;
    }
    roff += R;
    i = j;
  }
}
// After a barrier: row values (unit groups summed in order) to their runs, one thread per row.
QC_DEV void rows_finish(const Seg* sg, uint32_t nseg, uint32_t units, const float* part, uint32_t seq) {
  uint32_t R = 0;
  for (uint32_t k = 0; k < nseg; k++) R += sg[k].r1 - sg[k].r0;
  const uint32_t UG = unit_groups(units);
  for (uint32_t ri = threadIdx.x; ri < R; ri += blockDim.x) {
    uint32_t s = 0, first = 0;
    while (ri >= first + sg[s].r1 - sg[s].r0) {
      first += sg[s].r1 - sg[s].r0;
      s++;
    }
    float v = 0.f;
    for (uint32_t ug = 0; ug < UG; ug++) v += part[ug * R + ri];
    seg_emit(sg + s, sg[s].r0 + ri - first, v, seq);
  }
}

// Router rows of block c in whole 8-row groups (the first blocks hold them).  Measured: one row per
// block (128 blocks for a 128-expert F16 router) finishes the rows sooner but makes every block's
// gather of the 128 logits from 128 writers slower, a net loss.  rows: [b, e); bytes and src: the
// span to copy and its offset in the matrix.
struct RouterSlice {
  Span rows;
  uint32_t bytes;
  uint64_t src;
};
__host__ __device__ inline RouterSlice router_slice(const MatDesc& m, uint32_t nb, uint32_t c) {
  const Span g = span_of(groups_of(m.rows), nb, c);
  return {Span{g.b * 8, min(m.rows, g.e * 8)}, g.n() * m.group_bytes, (uint64_t)g.b * m.group_bytes};
}

// Position splits S and query-head groups GS of the attention for `time` positions: every
// (KV head, split, group) is one block.  The cost model is the per-block work: the score loop
// takes the same time for up to 4 query heads (a warp per position holds 4 in registers), the
// value sums grow with heads x positions, and each split adds a merge input.
__host__ __device__ inline void attn_split(uint32_t time, uint32_t G, uint32_t kvheads, uint32_t nb, uint32_t smax,
                                           uint32_t* S_out, uint32_t* GS_out, uint32_t* chunk_out) {
  uint32_t best = 0xffffffffu;
  for (uint32_t gs = 1; gs <= G && G % gs == 0; gs *= 2) {
    if (kvheads * gs > nb) break;
    uint32_t s = min(min(smax, nb / (kvheads * gs)), (time + kTokMinChunk - 1) / kTokMinChunk);
    s = s < 1 ? 1 : s;
    const uint32_t chunk = (time + s - 1) / s;
    s = (time + chunk - 1) / chunk;
    const uint32_t gh = G / gs;
    const uint32_t cost = chunk * ((gh + 3) / 4) * 4 + chunk * gh + (s > 1 ? 8 * s : 0);
    if (cost < best) {
      best = cost;
      *S_out = s;
      *GS_out = gs;
      *chunk_out = chunk;
    }
  }
}

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
  // small arrays: [keys E4*4][logits E][sel top][selw top][segments nsegs][residual rows][row outputs]
  const uint32_t E4 = (E + 3) / 4;
  uint8_t* mp = sm + T.misc_off;
  uint32_t* const key = reinterpret_cast<uint32_t*>(mp);
  uint32_t* const lsl = key;  // after the ranking: the selected slots this rank holds
  mp += E4 * 16;
  float* const lg = reinterpret_cast<float*>(mp);
  mp += up16(E * 4);
  uint32_t* const sel = reinterpret_cast<uint32_t*>(mp);
  mp += up16(top * 4);
  float* const selw = reinterpret_cast<float*>(mp);
  mp += up16(top * 4);
  Seg* const segs = reinterpret_cast<Seg*>(mp);
  mp += T.nsegs * sizeof(Seg);
  float* const part = reinterpret_cast<float*>(mp);  // unit-group partial sums of the row engine
  mp += up16(T.part_floats * 4);
  float* const qnw = reinterpret_cast<float*>(mp);  // [D] q_norm of the layer
  mp += up16(D * 4);
  float* const knw = reinterpret_cast<float*>(mp);  // [D] k_norm of the layer
  mp += up16(D * 4);
  float* const ropes = reinterpret_cast<float*>(mp);  // [D/2] (cos, sin) of this token's position
  mp += up16(D * 4);
  float* const xres = reinterpret_cast<float*>(mp);

  if (tid < sizeof(LayerDev) / 16) cp16(reinterpret_cast<uint8_t*>(&Ld[0]) + 16 * tid,
                                        reinterpret_cast<const uint8_t*>(&T.layers[0]) + 16 * tid);
  for (uint32_t i = tid; i < D / 4; i += TNT)  // the RoPE row of this position (the same in every layer)
    cp16(ropes + 4 * i, reinterpret_cast<const float*>(T.rope + (uint64_t)pos * (D / 2)) + 4 * i);
  cp_commit();
  if (tid == 0) {
    for (uint32_t i = 0; i < 2 + nslots; i++) mb_init(&mbar[i]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  cp_wait_all();
  __syncthreads();
  uint32_t parP = 0, parQ = 0;
  const uint32_t nbl = nb;
  // The ranks' MoE partials alternate between two halves by step parity: a rank one step ahead
  // writes the other half, and it can reach this half again only after every rank's previous
  // kernel (the one reading it) has ended.
  const uint64_t moe_half = T.ll_moe + (uint64_t)(seq & 1) * T.world * T.hidden;

  // ---- slices of this block (per layer; byte counts depend on the layer's formats) ----
  struct Slices {
    Span pq, pk, pv, so, sg, sd;
    RouterSlice rt;
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
    s.rt = router_slice(L.router, nbl, c);
    s.sg = span_of(top * groups_of(L.gate.rows), nbl, c);
    s.sd = span_of(groups_of(L.down.rows), nbl, c);
    s.bq = s.pq.n() * L.q.group_bytes;
    s.bk = s.pk.n() * L.k.group_bytes;
    s.bv = s.pv.n() * L.v.group_bytes;
    s.bA = s.bq + s.bk + s.bv;
    s.bO = s.so.n() * L.o.group_bytes;
    s.bR = s.rt.bytes;
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
    if (s.bR) bulk_copy(rQ + s.bO, L.router.w + s.rt.src, s.bR, &mbar[1]);
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
    prefetch_vectors(Ld[0], T.hidden, D);
  }

  // attention split of this token (the same for every layer): S position ranges of `chunk`
  // positions times GS groups of GH query heads per KV head, at most one block each
  const uint32_t time = pos + 1;
  uint32_t S = 1, GS = 1, chunk = time;
  attn_split(time, G, T.kvheads, nb, T.smax, &S, &GS, &chunk);
  const uint32_t GH = G / GS;
  const bool att = c < T.kvheads * S * GS;
  const uint32_t ah = att ? c / (S * GS) : 0, ags = att ? (c / S) % GS : 0, as = att ? c % S : 0;
  const uint32_t hq0 = ah * G + ags * GH;  // first query head of this block
  const uint32_t at0 = as * chunk, at1 = min(time, at0 + chunk);
  const float2* const cs = reinterpret_cast<const float2*>(ropes);
  const uint8_t* const erow = row_ptr(T.embd, T.embd.w, token);
  const __half* const edrow = drow_ptr(T.embd, T.embd.w, token);

  for (uint32_t l = 0; l < T.n_layers; l++) {
    const LayerDev& L = Ld[l & 1];
    const Slices s = slices(L);
    unsigned long long* const LL = T.ll + (uint64_t)l * T.ll_layer;
    // x of this layer: the previous layer's output (one rank), or its x' plus every rank's MoE partial
    const bool ep = T.world > 1;
    const unsigned long long* const Xin =
        l ? T.ll + (uint64_t)(l - 1) * T.ll_layer + (ep ? T.ll_xmid : T.ll_xout) : nullptr;
    const unsigned long long* const Xadd = l && ep ? T.ll + (uint64_t)(l - 1) * T.ll_layer + moe_half : nullptr;
    float* const kc_h = L.kc + (uint64_t)ah * T.ctx * D;
    float* const vc_h = L.vc + (uint64_t)ah * T.ctx * D;
    QC_TT(0);
    // next layer's descriptors into the other slot (last read in layer l-1)
    if (l + 1 < T.n_layers && tid < sizeof(LayerDev) / 16)
      cp16(reinterpret_cast<uint8_t*>(&Ld[(l + 1) & 1]) + 16 * tid,
           reinterpret_cast<const uint8_t*>(&T.layers[l + 1]) + 16 * tid);
    if (att)  // this layer's QK-norm weights, read in P2 (the previous layer's copies are consumed)
      for (uint32_t i = tid; i < D / 2; i += TNT) cp16(i < D / 4 ? qnw + 4 * i : knw + 4 * (i - D / 4),
                                                      (i < D / 4 ? L.q_norm + 4 * i : L.k_norm + 4 * (i - D / 4)));
    cp_commit();

    // ---- P1: Q, K, V = W rms(x, attn_norm) --------------------------------------------------
    const bool flA = uses_float_x(L.q.kind) || uses_float_x(L.k.kind) || uses_float_x(L.v.kind);
    if (tid == 0) {  // runs of Q, K and V rows (made visible by the staging barrier)
      segs[0] = make_seg(L.q, rP, s.pq.b * 8, min(L.q.rows, s.pq.e * 8), s.pq.b * 8, nullptr, nullptr,
                         LL + T.ll_qkv + s.pq.b * 8);
      segs[1] = make_seg(L.k, rP + s.bq, s.pk.b * 8, min(L.k.rows, s.pk.e * 8), s.pk.b * 8, nullptr, nullptr,
                         LL + T.ll_qkv + QD + s.pk.b * 8);
      segs[2] = make_seg(L.v, rP + s.bq + s.bk, s.pv.b * 8, min(L.v.rows, s.pv.e * 8), s.pv.b * 8, nullptr, nullptr,
                         LL + T.ll_qkv + QD + KD + s.pv.b * 8);
    }
    if (l == 0)
      stage_vectors<true>(
          stg, 1, T.hidden, L.q.units, flA, [&](uint32_t, uint32_t i) { return dequant_one(T.embd, erow, edrow, i); },
          L.attn_norm, T.eps, red);
    else
      stage_ll<true>(stg, 1, T.hidden, L.q.units, flA, Xin, L.attn_norm, T.eps, red, seq, st, l == 1, 20, Xadd,
                     ep ? T.world : 0);
    QC_TT(1);
    const XView xa = xview_at(stg, L.q.units, flA);
    if (s.bA) {
      mb_wait(&mbar[0], parP, st);
      parP ^= 1;
    }
    QC_TT(2);
    run_rows(segs, 3, L.q.units, xa, part);
    QC_TT(32);
    __syncthreads();
    rows_finish(segs, 3, L.q.units, part, seq);
    __syncthreads();  // staging area reused below
    QC_TT(3);

    // ---- P2: QK-norm, RoPE, KV append, split attention, merge --------------------------------
    if (att) {
      float* const qs = reinterpret_cast<float*>(stg);  // [GH][KP] this block's query heads
      float* const kn = qs + GH * KP;                   // [D] new key (normed, rotated)
      float* const vn = kn + D;                         // [D] new value
      float* const sc = vn + D;                         // [GH][kSub] scores, then weights
      float* const mls = sc + GH * kSub;                // [GH] running max, [GH] running sum, [GH] rescale
      const bool has_pos = at1 == time;
      // cached K/V rows of each step go to region P (free between P1 and P5), rows of D floats
      const uint32_t sub = min(kSub, T.p_bytes / (2 * D * 4));
      float* const ks = reinterpret_cast<float*>(rP);
      float* const vs = ks + sub * D;
      auto issue_kv = [&](uint32_t tb) {  // thread 0; returns nothing, copies rows [tb, min(tb + sub, at1, pos))
        const uint32_t te = min(min(tb + sub, at1), pos);
        if (te <= tb) return;
        const uint32_t bytes = (te - tb) * D * 4;
        proxy_fence();
        mb_expect(&mbar[0], 2 * bytes);
        bulk_copy(ks, kc_h + (uint64_t)tb * D, bytes, &mbar[0]);
        bulk_copy(vs, vc_h + (uint64_t)tb * D, bytes, &mbar[0]);
      };
      if (tid == 0) issue_kv(at0);
      QC_TT(26);
      ll_gather(LL + T.ll_qkv + (uint64_t)hq0 * D, GH * D,
                [&](uint32_t i, float v) { qs[(i / D) * KP + i % D] = v; }, seq, st);
      if (has_pos) {
        ll_gather(LL + T.ll_qkv + QD + (uint64_t)ah * D, D, [&](uint32_t i, float v) { kn[i] = v; }, seq, st);
        ll_gather(LL + T.ll_qkv + QD + KD + (uint64_t)ah * D, D, [&](uint32_t i, float v) { vn[i] = v; }, seq, st);
      }
      QC_TT(31);
      for (uint32_t g = tid; g < GH; g += TNT) {
        mls[g] = -INFINITY;
        mls[GH + g] = 0.f;
      }
      cp_wait_all();  // QK-norm weights
      __syncthreads();
      for (uint32_t g = warp; g < GH + (has_pos ? 1u : 0u); g += nw)  // the query heads, then the new key
        head_norm_rope(g < GH ? qs + g * KP : kn, g < GH ? qnw : knw, D, T.eps, cs);
      __syncthreads();
      if (has_pos && ags == 0 && warp == 0)  // model.rs:241-243: append k (normed, rotated) and v; one
        for (uint32_t i = lane; i < D; i += 32) {  // of the GS blocks holding this position writes the cache
          kc_h[(uint64_t)pos * D + i] = kn[i];
          vc_h[(uint64_t)pos * D + i] = vn[i];
        }
      QC_TT(24);
      // online softmax over steps of `sub` positions
      const float sd = sqrtf((float)D);
      // value accumulation: thread (head pair vg, 4 dims vd, position phase vt) sums positions t = vt mod VT
      const uint32_t D4 = D / 4, BT = (GH + 1) / 2 * D4;
      uint32_t VT = 1;
      while (VT * 2 * BT <= (uint32_t)TNT && VT < 16) VT *= 2;
      const uint32_t vt = tid / BT, vr = tid % BT, vg = vr / D4, vd = vr % D4, h0 = 2 * vg, h1 = 2 * vg + 1;
      const bool von = vt < VT && h0 < GH;
      float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f), acc1 = acc0;
      for (uint32_t tb = at0; tb < at1; tb += sub) {
        const uint32_t n = min(sub, at1 - tb);
        if (min(tb + n, pos) > tb) {  // cached rows of this step arrived
          mb_wait(&mbar[0], parP, st);
          parP ^= 1;
        }
        // s[g][t] = (q_g . k_t) / sqrt(D)  (ops.rs:84-91): a warp per position t, lanes over the
        // head dimension, 4 query heads at a time held in registers; the 4 partial dot products
        // are summed across the warp by a halving exchange (6 shuffles), leaving head (lane >> 3) & 3
        for (uint32_t gb = 0; gb < GH; gb += 4) {
          const uint32_t gn = min(4u, GH - gb);
          float4 qr[4][2];
#pragma unroll
          for (int g = 0; g < 4; g++)
#pragma unroll
            for (int i = 0; i < 2; i++) {
              const uint32_t j = lane + 32 * i;
              qr[g][i] = (g < (int)gn && j < D4) ? reinterpret_cast<const float4*>(qs + (gb + g) * KP)[j]
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
          for (uint32_t t = warp; t < n; t += nw) {
            const float4* k4 = reinterpret_cast<const float4*>(tb + t == pos ? kn : ks + t * D);
            float p[4];
#pragma unroll
            for (int g = 0; g < 4; g++) p[g] = 0.f;
#pragma unroll
            for (int i = 0; i < 2; i++) {
              const uint32_t j = lane + 32 * i;
              if (j < D4) {
                const float4 a = k4[j];
#pragma unroll
                for (int g = 0; g < 4; g++) {
                  p[g] = fmaf(a.x, qr[g][i].x, p[g]);
                  p[g] = fmaf(a.y, qr[g][i].y, p[g]);
                  p[g] = fmaf(a.z, qr[g][i].z, p[g]);
                  p[g] = fmaf(a.w, qr[g][i].w, p[g]);
                }
              }
            }
            // halving exchange: 4 partial sums per lane -> head (lane >> 3) & 3 summed over the warp
            const bool b4 = lane & 16, b3 = lane & 8;
            float h2[2];
#pragma unroll
            for (int k = 0; k < 2; k++) {
              const float send = b4 ? p[k] : p[k + 2], keep = b4 ? p[k + 2] : p[k];
              h2[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
            }
            float h1v;
            {
              const float send = b3 ? h2[0] : h2[1], keep = b3 ? h2[1] : h2[0];
              h1v = keep + __shfl_xor_sync(0xffffffffu, send, 8);
            }
            h1v += __shfl_xor_sync(0xffffffffu, h1v, 4);
            h1v += __shfl_xor_sync(0xffffffffu, h1v, 2);
            h1v += __shfl_xor_sync(0xffffffffu, h1v, 1);
            const uint32_t g = (lane >> 3) & 3;
            if ((lane & 7) == 0 && g < gn) sc[(gb + g) * kSub + t] = h1v / sd;
          }
        }
        __syncthreads();
        for (uint32_t g = warp; g < GH; g += nw) {
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
            mls[2 * GH + g] = f;
            mls[GH + g] = mls[GH + g] * f + sum;
            mls[g] = mn;
          }
        }
        __syncthreads();
        // acc[h][4 dims] = sum_t p[h][t] v_t; thread (pair of heads h0 = 2 vg, h1 = h0 + 1; 4 dims vd)
        if (von) {
          const bool two = h1 < GH;
          const float f0 = mls[2 * GH + h0], f1 = two ? mls[2 * GH + h1] : 0.f;
          acc0.x *= f0;
          acc0.y *= f0;
          acc0.z *= f0;
          acc0.w *= f0;
          acc1.x *= f1;
          acc1.y *= f1;
          acc1.z *= f1;
          acc1.w *= f1;
          const float* p0 = sc + h0 * kSub;
          const float* p1 = sc + (two ? h1 : h0) * kSub;
          for (uint32_t t = vt; t < n; t += VT) {
            const float4 v = *reinterpret_cast<const float4*>((tb + t == pos ? vn : vs + t * D) + 4 * vd);
            const float a = p0[t], b = two ? p1[t] : 0.f;
            acc0.x = fmaf(a, v.x, acc0.x);
            acc0.y = fmaf(a, v.y, acc0.y);
            acc0.z = fmaf(a, v.z, acc0.z);
            acc0.w = fmaf(a, v.w, acc0.w);
            acc1.x = fmaf(b, v.x, acc1.x);
            acc1.y = fmaf(b, v.y, acc1.y);
            acc1.z = fmaf(b, v.z, acc1.z);
            acc1.w = fmaf(b, v.w, acc1.w);
          }
        }
        __syncthreads();
        if (tid == 0 && tb + sub < at1) issue_kv(tb + sub);
      }
      {  // partial sums of the position phases through region P (its K/V rows are consumed), in order
        float4* const va = reinterpret_cast<float4*>(rP);  // [VT][BT][2]
        if (von) {
          va[(vt * BT + vr) * 2] = acc0;
          va[(vt * BT + vr) * 2 + 1] = acc1;
        }
        __syncthreads();
        if (von && vt == 0)
          for (uint32_t k = 1; k < VT; k++) {
            const float4 a = va[(k * BT + vr) * 2], b = va[(k * BT + vr) * 2 + 1];
            acc0.x += a.x;
            acc0.y += a.y;
            acc0.z += a.z;
            acc0.w += a.w;
            acc1.x += b.x;
            acc1.y += b.y;
            acc1.z += b.z;
            acc1.w += b.w;
          }
      }
      QC_TT(25);
      for (uint32_t hh = 0; hh < 2 && von && vt == 0; hh++) {
        const uint32_t ag = h0 + hh;
        if (ag >= GH) continue;
        const float4 acc = hh ? acc1 : acc0;
        if (S == 1) {  // one split: normalize and publish the output directly
          const float inv = 1.f / mls[GH + ag];
          unsigned long long* o = LL + T.ll_attn + (uint64_t)(hq0 + ag) * D + 4 * vd;
          ll_put2(o, acc.x * inv, acc.y * inv, seq);
          ll_put2(o + 2, acc.z * inv, acc.w * inv, seq);
        } else {  // partial state [acc[D], m, l] of (head, split)
          unsigned long long* o = LL + T.ll_part + ((uint64_t)(hq0 + ag) * T.smax + as) * (D + 2);
          ll_put2(o + 4 * vd, acc.x, acc.y, seq);
          ll_put2(o + 4 * vd + 2, acc.z, acc.w, seq);
          if (vd == 0) ll_put2(o + D, mls[ag], mls[GH + ag], seq);
        }
      }
      if (S > 1) {  // this split merges heads hq0 + as, hq0 + as + S, ... of its head group
        float* const pb = reinterpret_cast<float*>(stg);  // [S][D + 2]
        float* const fw = pb + S * (D + 2);               // [S]
        for (uint32_t gl = as; gl < GH; gl += S) {
          const uint32_t g = hq0 + gl;
          __syncthreads();
          ll_gather(LL + T.ll_part + (uint64_t)g * T.smax * (D + 2), S * (D + 2),
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
            ll_put(LL + T.ll_attn + (uint64_t)g * D + d, o * red[0], seq);
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
      if (l == 0) xres[r - or0] = dequant_one(T.embd, erow, edrow, r);
      else {
        float v = ll_wait1(Xin + r, seq, st);
        for (uint32_t q = 0; ep && q < T.world; q++) v = __fadd_rn(v, ll_wait1_sys(Xadd + (uint64_t)q * T.hidden + r, seq, st));
        xres[r - or0] = v;
      }
    if (tid == 0) segs[0] = make_seg(L.o, rQ, or0, or1, or0, xres, nullptr, LL + T.ll_xmid + or0);
    stage_ll<false>(stg, 1, QD, L.o.units, flO, LL + T.ll_attn, nullptr, 0.f, red, seq, st, l == 1, 21);
    QC_TT(5);
    if (s.bOR) {
      mb_wait(&mbar[1], parQ, st);
      parQ ^= 1;
    }
    run_rows(segs, 1, L.o.units, xview_at(stg, L.o.units, flO), part);
    QC_TT(33);
    __syncthreads();
    rows_finish(segs, 1, L.o.units, part, seq);
    __syncthreads();
    QC_TT(6);

    // ---- P4: router logits of rms(x', ffn_norm) (the same vector feeds gate/up) ----------------
    const bool flR = uses_float_x(L.router.kind) || uses_float_x(L.gate.kind) || uses_float_x(L.up.kind);
    if (tid == 0) {
      const uint32_t r0 = s.rt.rows.b;
      segs[0] = make_seg(L.router, rQ + s.bO, r0, s.rt.rows.e, r0, nullptr, nullptr, LL + T.ll_rl + r0);
    }
    stage_ll<true>(stg, 1, T.hidden, L.router.units, flR, LL + T.ll_xmid, L.ffn_norm, T.eps, red, seq, st, l == 1, 22);
    const XView xf = xview_at(stg, L.router.units, flR);
    QC_TT(7);
    run_rows(segs, 1, L.router.units, xf, part);
    QC_TT(39);
    __syncthreads();
    rows_finish(segs, 1, L.router.units, part, seq);
    QC_TT(8);

    // ---- P5: top-k with ties to the lower index + softmax over the kept logits, gate/up + SwiGLU
    ll_gather(LL + T.ll_rl, E, [&](uint32_t i, float v) {
      lg[i] = v;
      key[i] = total_key_u(v);
    }, seq, st);
    for (uint32_t e = E + tid; e < 4 * E4; e += TNT) key[e] = 0;  // below every real key: never counted
    __syncthreads();
    QC_TT(27);
    {  // rank of each logit (ties to the lower index), 4 threads per expert reading 4 keys at a time
      for (uint32_t base = 0; base < E; base += TNT / 4) {
        const uint32_t e = base + tid / 4, part = tid % 4;
        uint32_t rank = 0;
        if (e < E) {
          const uint32_t ke = key[e];
          for (uint32_t i = part; i < E4; i += 4) {
            const uint4 k4 = reinterpret_cast<const uint4*>(key)[i];
            const uint32_t j = 4 * i;
            rank += (k4.x > ke || (k4.x == ke && j < e)) + (k4.y > ke || (k4.y == ke && j + 1 < e)) +
                    (k4.z > ke || (k4.z == ke && j + 2 < e)) + (k4.w > ke || (k4.w == ke && j + 3 < e));
          }
        }
        rank += __shfl_xor_sync(0xffffffffu, rank, 1);
        rank += __shfl_xor_sync(0xffffffffu, rank, 2);
        if (e < E && part == 0) {
          if (rank < top) sel[rank] = e;
          if (c == 0 && !isfinite(lg[e])) atomicOr(&st->nonfinite, 1u);
        }
      }
    }
    __syncthreads();
    QC_TT(28);
    // The selected experts this rank holds (all of them on one rank), in selection order: bit k of
    // `mine` for slot k (top <= 32).  Each warp derives them itself, so the copies of their rows are
    // issued by several warps at once right after the ranking.
    const uint32_t mine = __ballot_sync(0xffffffffu, lane < top && sel[lane] - T.e_lo < T.e_n);
    const uint32_t nl = __popc(mine);
    const uint32_t gi = groups_of(L.gate.rows), gub = L.gate.group_bytes + L.up.group_bytes;
    const Span sgd = span_of(nl * gi, nbl, c);  // this block's (local expert, gate/up row group) items
    const uint32_t nitem = sgd.n(), bGUd = nitem * gub, bDd = nl * s.sd.n() * L.down.group_bytes;
    // runs of items: one per local expert the span touches; run r covers items [i0, i1)
    const uint32_t nruns = nitem ? (sgd.e - 1) / gi - sgd.b / gi + 1 : 0;
    auto run_of = [&](uint32_t r, uint32_t* i0, uint32_t* i1) {
      *i0 = r ? (sgd.b / gi + r) * gi : sgd.b;
      *i1 = min((*i0 / gi + 1) * gi, sgd.e);
    };
    float* const gout = xres;  // [2][nitem * 8] gate then up results
    if (warp == 0) {
      // ops.rs:29-44 in selection order: max, exp, sequential sum, divide
      const float v = lane < top ? lg[sel[lane]] : -INFINITY;
      const float mx = warp_max(v);
      const float ex = lane < top ? expf(v - mx) : 0.f;
      float sum = 0.f;
      for (uint32_t k = 0; k < top; k++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, ex, k));
      if (lane < top) selw[lane] = ex / sum;
      if ((mine >> lane) & 1u) lsl[__popc(mine & ((1u << lane) - 1u))] = lane;
      QC_TT(29);
    } else if (warp == 1) {  // their gate/up rows into P (Q/K/V and K/V rows consumed): run r, gate or up;
      if (lane < 2 * nruns) {
        uint32_t i0, i1;
        run_of(lane >> 1, &i0, &i1);
        const uint32_t e = sel[__fns(mine, 0, (int)(i0 / gi) + 1)] - T.e_lo;
        const MatDesc& m = lane & 1u ? L.up : L.gate;
        proxy_fence();
        bulk_copy(rP + (i0 - sgd.b) * gub + (lane & 1u) * (i1 - i0) * L.gate.group_bytes,
                  m.w + (uint64_t)e * m.expert_stride + (uint64_t)(i0 % gi) * m.group_bytes, (i1 - i0) * m.group_bytes,
                  &mbar[0]);
      }
      if (lane == 0 && bGUd) mb_expect(&mbar[0], bGUd);
      __syncwarp();
      // then the down rows of every local selected expert into Q (needed one exchange later)
      if (lane < nl && bDd) {
        const uint32_t per = s.sd.n() * L.down.group_bytes;
        proxy_fence();
        bulk_copy(rQ + lane * per,
                  L.down.w + (uint64_t)(sel[__fns(mine, 0, (int)lane + 1)] - T.e_lo) * L.down.expert_stride +
                      (uint64_t)s.sd.b * L.down.group_bytes,
                  per, &mbar[1]);
      }
      if (lane == 0 && bDd) mb_expect(&mbar[1], bDd);
    } else if (warp == 3 && lane < nruns) {  // row runs: all gate runs, then all up runs (one format per call)
      uint32_t i0, i1;
      run_of(lane, &i0, &i1);
      const uint32_t r0 = (i0 % gi) * 8, r1 = min(L.gate.rows, (i0 % gi + i1 - i0) * 8), it0 = i0 - sgd.b;
      uint8_t* const base = rP + it0 * gub;
      segs[lane] = make_seg(L.gate, base, r0, r1, r0, nullptr, gout + it0 * 8, nullptr);
      segs[nruns + lane] =
          make_seg(L.up, base + (i1 - i0) * L.gate.group_bytes, r0, r1, r0, nullptr, gout + (nitem + it0) * 8, nullptr);
    }
    __syncthreads();
    QC_TT(9);
    if (bGUd) {
      mb_wait(&mbar[0], parP, st);
      parP ^= 1;
    }
    QC_TT(10);
    run_rows(segs, 2 * nruns, L.gate.units, xf, part);
    QC_TT(34);
    __syncthreads();
    rows_finish(segs, 2 * nruns, L.gate.units, part, seq);
    __syncthreads();
    QC_TT(35);
    for (uint32_t idx = tid; idx < nitem * 8; idx += TNT) {
      const uint32_t i = sgd.b + idx / 8, slot = i / gi, r = (i % gi) * 8 + idx % 8;  // slot: index into lsl
      if (r < T.inter) {
        const float gv = gout[idx], uv = gout[nitem * 8 + idx];
        ll_put(LL + T.ll_h + (uint64_t)slot * T.inter + r, __fmul_rn(gv / (1.f + expf(-gv)), uv), seq);
      }
    }
    QC_TT(36);
    cp_wait_all();  // the next layer's descriptors
    __syncthreads();
    if (tid == 0) {  // region P is free: next layer's Q/K/V slice, or the first vocab stages
      if (l + 1 < T.n_layers) prefetch_vectors(Ld[(l + 1) & 1], T.hidden, D);
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
    {
      const uint32_t pbytes = s.sd.n() * L.down.group_bytes;
      for (uint32_t k = tid; k < nl; k += TNT)
        segs[k] = make_seg(L.down, rQ + k * pbytes, dr0, dr1, dr0, nullptr, dout + k * nd, nullptr);
    }
    stage_ll<false>(stg, nl, T.inter, L.down.units, flD, LL + T.ll_h, nullptr, 0.f, red, seq, st, l == 1, 23);
    QC_TT(12);
    const uint32_t xb = xview_bytes(L.down.units, flD);
    if (bDd) {
      mb_wait(&mbar[1], parQ, st);
      parQ ^= 1;
    }
    QC_TT(13);
    const uint32_t dpart = unit_groups(L.down.units) * (dr1 > dr0 ? dr1 - dr0 : 0);
    if (dr1 > dr0 && nl) {
      const uint32_t per = nw >= nl ? nw / nl : 1;
      for (uint32_t k = warp / per; k < nl; k += nw / per)
        run_rows(segs + k, 1, L.down.units, xview_at(stg + k * xb, L.down.units, flD), part + k * dpart, warp % per,
                 per);
    }
    QC_TT(37);
    __syncthreads();
    {  // every (expert, row) pair at once: unit groups summed in order into dout
      const uint32_t R = dr1 > dr0 ? dr1 - dr0 : 0, UG = unit_groups(L.down.units);
      for (uint32_t i = tid; i < nl * R; i += TNT) {
        const uint32_t k = i / R, ri = i % R;
        const float* pp = part + k * dpart + ri;
        float v = 0.f;
        for (uint32_t ug = 0; ug < UG; ug++) v += pp[ug * R];
        dout[k * nd + ri] = v;
      }
    }
    __syncthreads();
    QC_TT(38);
    for (uint32_t r = dr0 + tid; r < dr1; r += TNT) {
      float acc = 0.f;
      for (uint32_t k = 0; k < nl; k++) acc = __fadd_rn(acc, __fmul_rn(selw[lsl[k]], dout[k * nd + r - dr0]));
      if (!ep) ll_put(LL + T.ll_xout + r, __fadd_rn(dres[r - dr0], acc), seq);
      else  // this rank's share of moe, into every rank's exchange buffer
        for (uint32_t q = 0; q < T.world; q++)
          ll_put_sys(T.peers[q] + (uint64_t)l * T.ll_layer + moe_half + (uint64_t)T.rank * T.hidden + r, acc, seq);
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
  stage_ll<true>(stg, 1, T.hidden, mo.units, flV,
                 T.ll + (uint64_t)(T.n_layers - 1) * T.ll_layer + (T.world > 1 ? T.ll_xmid : T.ll_xout), T.out_norm,
                 T.eps, red, seq, st, false, 0, T.world > 1 ? T.ll + (uint64_t)(T.n_layers - 1) * T.ll_layer + moe_half : nullptr,
                 T.world > 1 ? T.world : 0);
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
  if (d.top > 32) return "more than 32 experts per token";
  TokenPlan t{};
  t.nb = nb;
  t.smax = std::max(1u, std::min(nb / d.kvheads, (d.ctx + kTokMinChunk - 1) / kTokMinChunk));
  const uint32_t cap = std::min<uint32_t>(g_token_smem_cap, (uint32_t)max_smem);
  uint32_t P = 0, Q = 0, stage = 0, res = 0, outs = 0, runs = 1, partf = 0;
  const AttnSmem as = attn_stage_bytes(G, D, t.smax);
  stage = std::max(as.attn, as.merge);
  for (uint32_t l = 0; l < a.n_layers; l++) {
    const LayerDev& L = a.layers[l];
    if (L.q.units != L.k.units || L.q.units != L.v.units || L.router.units != L.gate.units || L.gate.units != L.up.units ||
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
      const Span so = span_of(groups_of(L.o.rows), nb, c);
      const RouterSlice rt = router_slice(L.router, nb, c);
      const Span sg = span_of(d.top * groups_of(L.gate.rows), nb, c), sd = span_of(groups_of(L.down.rows), nb, c);
      const uint32_t bOR = so.n() * L.o.group_bytes + rt.bytes;
      const uint32_t bGU = sg.n() * (L.gate.group_bytes + L.up.group_bytes);
      const uint32_t bD = sd.n() * d.top * L.down.group_bytes;
      P = std::max(P, std::max(bA, bGU));
      Q = std::max(Q, std::max(bOR, bD));
      res = std::max(res, std::max(so.n() * 8, sd.n() * 8));
      {  // unit-group partial sums of each phase's rows
        auto ug = [](uint32_t units) { return (units + 7) / 8; };
        uint32_t ra = 0;
        for (int k = 0; k < 3; k++) {
          const uint32_t lo = std::max(sa.b, seg0[k]), hi = std::min(sa.e, seg0[k] + segn[k]);
          if (hi > lo) ra += (hi - lo) * 8;
        }
        partf = std::max(partf, ug(L.q.units) * ra);
        partf = std::max(partf, ug(L.o.units) * so.n() * 8);
        partf = std::max(partf, ug(L.router.units) * rt.rows.n());
        partf = std::max(partf, ug(L.gate.units) * 2 * sg.n() * 8);
        partf = std::max(partf, d.top * ug(L.down.units) * sd.n() * 8);
      }
      {  // gate/up runs (one per selected expert the block's items touch)
        const uint32_t gi = groups_of(L.gate.rows);
        uint32_t n = 0;
        for (uint32_t i = sg.b; i < sg.e; n++) i += std::min(gi - i % gi, sg.e - i);
        runs = std::max(runs, n);
      }
      outs = std::max(outs, std::max(2 * sg.n() * 8, (d.top + 1) * sd.n() * 8));
    }
  }
  stage = std::max(stage, xview_bytes(a.out.units, uses_float_x(a.out.kind)));
  // vocab stages: up to 4 groups (32 rows: two per warp) and 56 KB each, at least two slots over P
  // and Q (measured on the standalone matvec: 32-row stages stream the Q6_K vocab rows ~15% faster
  // than 24-row ones, the per-stage work between barriers being the limit)
  const uint32_t ogb = a.out.group_bytes;
  const uint32_t vper = (groups_of(a.out.rows) + nb - 1) / nb;
  uint32_t sg = std::max(1u, std::min(std::min(57344u / ogb, 4u), (vper + 1) / 2));
  const uint32_t slot = sg * ogb;
  P = std::max(P, slot);
  Q = std::max(Q, slot);
  // attention stages its cached K/V rows in P: at least 8 positions, up to kSub when room is left
  const uint32_t kv_pos = 2 * D * 4;
  P = std::max(std::max(P, 8 * kv_pos), 16384u);  // (also the attention's partial value sums)
  P = up16(P);
  Q = up16(Q);
  t.nsegs = std::max(std::max(3u, d.top), 2 * runs);
  t.nsegs += t.nsegs & 1;
  t.part_floats = partf;
  const uint32_t misc = (d.experts + 3) / 4 * 16 + up16(d.experts * 4) + 2 * up16(d.top * 4) +
                        t.nsegs * (uint32_t)sizeof(Seg) + up16(partf * 4) + 3 * up16(D * 4) +
                        up16(std::max(res, outs) * 4);
  const uint32_t total = P + Q + up16(stage) + misc;
  if (total > cap) return "the per-block weight slices and staging exceed the shared memory of one SM";
  if (P < kSub * kv_pos) P += std::min(cap - total, kSub * kv_pos - P) & ~15u;
  t.out_sg = sg;
  t.nsp = std::min(P / slot, kMaxTokenSlots / 2);
  t.nsq = std::min(Q / slot, kMaxTokenSlots - t.nsp);
  t.p_bytes = P;
  t.q_bytes = Q;
  t.stage_off = P + Q;
  t.misc_off = t.stage_off + up16(stage);
  t.smem = t.misc_off + misc;
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
  t.ll_moe = o;  // [2][world][hidden] partial MoE vectors written by the ranks (expert parallelism)
  o += a.ep_world > 1 ? ev(2ull * a.ep_world * d.hidden) : 0;
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
  T.nsegs = p.nsegs;
  T.world = a.ep_world ? a.ep_world : 1;
  T.rank = a.ep_rank;
  T.e_lo = a.e_lo;
  T.e_n = a.e_n ? a.e_n : d.experts;
  T.peers = a.peers;
  T.ll_moe = p.ll_moe;
  T.part_floats = p.part_floats;
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
