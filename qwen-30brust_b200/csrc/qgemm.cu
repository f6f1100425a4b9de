// Tensor-core GEMM over GGUF K-quant rows: y[n][r] = sum_k W[r][k] x_n[k] for a batch of activation
// vectors, W in Q4_K or Q6_K (the engine's 8-row-group device layout), on the 5th-generation tensor
// cores (tcgen05.mma kind::f16, fp32 accumulators in TMEM).  It replaces the reference's per-vector
// Backend::matvec (backend.rs:28-52) wherever several vectors meet the same rows: the batched
// attention projections and vocabulary rows of several sequences, and the grouped expert GEMMs of a
// MoE layer (model.rs:249-287 for a batch of tokens).
//
// Exact operands.  A K-quant weight is d * sc * q (- dmin * mn for Q4_K) with small integers sc, q, mn
// (quant.rs:50-77).  The A operand holds the integers only, exact in fp16:
//   Q4_K  sc * q  (<= 63 * 15), one plane;
//   Q6_K  sc * (q - 32) (|.| <= 4096) as hi = fp16(sc * (q - 32)) and lo = the remainder (0 or +-1),
// and each 256-element super-block b accumulates into its own TMEM columns, so the per-block factor
// d_b is applied once in the epilogue: y = sum_b d_b * acc_b.  The Q4_K min term
// -sum_j dmin * mn_j * (sum of the 32 x of sub-block j) is one extra K = 16 step per super-block into
// a separate accumulator: A = (dmin * mn_j * s_min) as fp16 hi | lo, B = the sub-block sums.
// Activations come as a "B image" built once per batch (qg_image): x * hs (hs a power of two per
// vector) as fp16 hi + lo planes in the layout the MMAs read, so a B stage is two bulk copies.
// Products keep ~22 significant bits (A exact, B hi + lo); the only other rounding is the fp32
// accumulation, so results stay within the matvec tolerance of the reference's f32 fold.
//
// Structure: a persistent CTA per SM (384 threads) walks work items (group, 128-row tile, pass of up
// to NP vectors).  Warp 0 brings raw weight rows into a ring of shared-memory stages with bulk copies
// (one stage = one super-block of 128 rows); warp 2 brings B stages; warps 4-11 turn raw rows into
// A stages (one per K step of 64) and run the epilogue; warp 1 issues the MMAs (one elected thread)
// and commits them to the stages' mbarriers.  Every wait is bounded (2 s): a timed-out role sets an
// error bit, the others stop at their next wait, and copies and MMAs in flight are drained before the
// accumulator is released.
#include <cuda_fp16.h>

#include "kernels.h"

namespace qc {
namespace {

constexpr uint32_t kThreads = 384;
constexpr uint32_t kProdWarp0 = 4;  // warps 4..11 produce A and run the epilogue
constexpr uint32_t kProd = 256;     // producer threads
constexpr unsigned long long kWaitNs = 2000000000ull;
constexpr uint32_t kNone = 0xffffffffu;

template <int AK>
struct Cfg;
template <>
struct Cfg<Q4_K> {  // KS: K steps of 64 per stage; kcsA: 16-byte chunks per A row in a stage (+2: min)
  static constexpr uint32_t blk = 144, RS = 3, planes = 1, KS = 2, kcsA = 8 * KS + 2;
};
template <>
struct Cfg<Q6_K> {
  static constexpr uint32_t blk = 208, RS = 3, planes = 2, KS = 1, kcsA = 8;
};
constexpr uint32_t kMaxSS = 8;  // stages (runtime count a.SS: qgemm_shape)
template <int AK>
constexpr uint32_t a_stage_bytes() {
  return Cfg<AK>::planes * 128 * Cfg<AK>::kcsA * 16;
}

QC_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
QC_DEV unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
QC_DEV void mbar_init(uint64_t* m, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(m)), "r"(count) : "memory");
}
QC_DEV void mbar_arrive(uint64_t* m) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(m)) : "memory");
}
QC_DEV void mbar_expect(uint64_t* m, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(m)), "r"(bytes) : "memory");
}
QC_DEV void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* m) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(m))
               : "memory");
}
// Wait (at most 2 s, or until another role gave up) for the phase with the given parity.
QC_DEV bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
QC_DEV bool mbar_wait(uint64_t* m, uint32_t parity, volatile int* abort_flag) {
  const uint32_t a = smem_u32(m);
  if (mbar_try(a, parity)) return true;  // (the common case: no clock read)
  const unsigned long long t0 = now_ns();
  for (uint32_t i = 0;; i++) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 255) == 255) {
      if (*abort_flag) return false;
      if (now_ns() - t0 > kWaitNs) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}
// A ring of n stages: the slot and phase parity of the current use, advanced without division.
struct Ring {
  uint32_t n, slot, phase;
  QC_DEV explicit Ring(uint32_t stages) : n(stages), slot(0), phase(0) {}
  QC_DEV void next() {
    if (++slot == n) {
      slot = 0;
      phase ^= 1;
    }
  }
};
// Drain: wait (bounded) for a phase, ignoring the abort flag.
QC_DEV void mbar_drain(uint64_t* m, uint32_t parity) {
  int never = 0;
  mbar_wait(m, parity, &never);
}
// Barrier of the 8 producer warps on an mbarrier (count 8), so that a warp which gave up makes the
// others' wait time out instead of blocking: false if it did.
QC_DEV bool prod_sync(uint64_t* b, uint32_t* phase, volatile int* abort_flag) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(b);
  const bool ok = mbar_wait(b, *phase & 1, abort_flag);
  ++*phase;
  __syncwarp();
  return ok;
}

QC_DEV unsigned long long sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (unsigned long long)((addr >> 4) & 0x3fff) | ((unsigned long long)((lbo >> 4) & 0x3fff) << 16) |
         ((unsigned long long)((sbo >> 4) & 0x3fff) << 32) | (1ull << 46);
}
// D (+)= A B: mma_first overwrites D, mma_acc adds to it.
QC_DEV void mma_first(uint32_t d, unsigned long long a, unsigned long long b, uint32_t idesc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, 0, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc)
      : "memory");
}
QC_DEV void mma_acc(uint32_t d, unsigned long long a, unsigned long long b, uint32_t idesc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.eq.b32 p, 0, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc)
      : "memory");
}
QC_DEV void mma_commit(uint64_t* m) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(m))
               : "memory");
}

QC_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
QC_DEV uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
QC_DEV __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// x as fp16 hi + lo (x = hi + lo to ~22 bits when |x| < 2^15), two values per word.
QC_DEV void split2(float a, float b, uint32_t* hi, uint32_t* lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 back = __half22float2(h);
  *hi = h2u(h);
  *lo = h2u(__floats2half2_rn(a - back.x, b - back.y));
}

// Item -> (group, tile, pass).  Groups are ordered by first item; an empty group shares its first
// item with the next one, so the group of item i is the last one starting at or before i.
struct Item {
  uint32_t g, tile, n0, N, nn;
};
constexpr uint32_t kMaxGroups = 1024;
QC_DEV const QgGroup& group_at(const QgArgs& a, uint32_t g) { return a.groups ? a.groups[g] : a.inl[g]; }
// (item0 of every group is staged in shared memory: g0[])
QC_DEV Item decode_item(const QgArgs& a, const uint32_t* g0, uint32_t i) {
  uint32_t lo = 0, hi = a.ngroups - 1;
  while (lo < hi) {
    const uint32_t mid = (lo + hi + 1) >> 1;
    if (g0[mid] <= i) lo = mid;
    else hi = mid - 1;
  }
  const QgGroup& g = group_at(a, lo);
  const uint32_t passes = (g.nimg + a.NP - 1) / a.NP, local = i - g.item0;
  Item it;
  it.g = lo;
  it.tile = local / passes;
  it.n0 = (local % passes) * a.NP;
  it.N = min(a.NP, g.nimg - it.n0);
  it.nn = g.cnt > it.n0 ? min(it.N, g.cnt - it.n0) : 0;
  return it;
}
// Row r (< 128) of an item's tile: its matrix and row there, or false past the matrix.
QC_DEV bool tile_row(const QgArgs& a, uint32_t mat, uint32_t tile, uint32_t r, uint32_t* mi, uint32_t* row) {
  if (a.pair) {
    *mi = mat + (r >> 6);
    *row = tile * 64 + (r & 63);
  } else {
    *mi = mat;
    *row = tile * 128 + r;
  }
  return *row < a.mats[*mi].rows;
}
// What the loaders and the MMA issuer need of an item, read one item ahead.
struct ItemDesc {
  uint32_t tile, n0, N, nimg, imgoff, mat, e;
};
QC_DEV ItemDesc load_item(const QgArgs& a, const uint32_t* g0, uint32_t i) {
  const Item it = decode_item(a, g0, i);
  const QgGroup& g = group_at(a, it.g);
  return ItemDesc{it.tile, it.n0, it.N, g.nimg, g.imgoff, g.mat, g.e};
}

// Image layout.  K steps of 64 columns; with min chunks (Q4_K activations), the last K step of each
// super-block carries two more 16-byte chunks (the sub-block sums).  Per K step: [plane hi, lo]
// [row / 8][chunk][row % 8][16 bytes].
QC_DEV uint32_t kcs_of(uint32_t s, uint32_t hasmin) { return 8 + ((hasmin && (s & 3) == 3) ? 2 : 0); }
QC_DEV uint32_t kc_before(uint32_t s, uint32_t hasmin) { return 8 * s + (hasmin ? 2 * (s >> 2) : 0); }

template <int AK, int EPI>
__global__ void __launch_bounds__(kThreads, 1) k_qgemm(const __grid_constant__ QgArgs a) {
  using C = Cfg<AK>;
  extern __shared__ __align__(1024) uint8_t sm_raw[];
  // (tensor copies want 128-byte aligned destinations: the carve-up starts at a 1024-byte boundary)
  uint8_t* sm = sm_raw + ((1024 - (smem_u32(sm_raw) & 1023)) & 1023);
  __shared__ __align__(8) uint64_t raw_full[C::RS], raw_empty[C::RS], st_full[kMaxSS], st_empty[kMaxSS], acc_full,
      psync;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ uint32_t g0[kMaxGroups];
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t K = a.K, S = K / 64, nsb = K / 256;
  const bool hasminA = AK == Q4_K;
  const uint32_t nitems = a.nitems_dev ? *a.nitems_dev : a.nitems;
  // shared-memory carve-up (the host sizes it with qgemm_smem)
  const uint32_t kcsB = a.img_hasmin ? 10 : 8;
  // a raw stage: two (64-row tile, super-block) blocks of the GEMM layout (rows 0-63, 64-127)
  const uint32_t half_bytes = 64 * (AK == Q4_K ? 144 : 210), raw_bytes = 2 * half_bytes;
  // a stage: the A operand of KS K steps, then for each of them the B planes (hi, lo) of the pass
  const uint32_t a_part = a_stage_bytes<AK>(), b_sub = 2 * a.NP * kcsB * 16, stage_bytes = a_part + C::KS * b_sub;
  uint8_t* raw = sm;
  uint8_t* stg = raw + C::RS * raw_bytes;
  const uint32_t SS = a.SS;
  float* dsm = reinterpret_cast<float*>(stg + SS * stage_bytes);  // [part][nsb][128] d of each row
  float* hsm = dsm + 2 * nsb * 128;                              // [2][NP] 1 / scale of each vector
  uint32_t* ysm = reinterpret_cast<uint32_t*>(hsm + 2 * a.NP);  // [2][NP] output row of each vector
  const uint32_t img_row = 32 * kc_before(S, a.img_hasmin);     // image bytes per vector

  for (uint32_t g = tid; g < a.ngroups; g += kThreads) g0[g] = group_at(a, g).item0;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_base))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    abort_flag = 0;
    for (uint32_t i = 0; i < C::RS; i++) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kProd / 32);
    }
    for (uint32_t i = 0; i < SS; i++) {
      mbar_init(&st_full[i], kProd / 32 + 1);  // the producer warps and the B copier (with the bytes)
      mbar_init(&st_empty[i], 1);
    }
    mbar_init(&acc_full, 1);
    mbar_init(&psync, kProd / 32);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  volatile int* ab = &abort_flag;

  if (warp == 0) {
    // ---- raw weight rows: one stage per (item, super-block): two contiguous bulk copies ----
    uint32_t ctr = 0;
    Ring ring(C::RS);
    bool ok = true;
    ItemDesc nx{};
    if (blockIdx.x < nitems) nx = load_item(a, g0, blockIdx.x);
    for (uint32_t i = blockIdx.x; i < nitems && ok; i += gridDim.x) {
      const ItemDesc it = nx;
      if (i + gridDim.x < nitems) nx = load_item(a, g0, i + gridDim.x);
      for (uint32_t b = 0; b < nsb; b++, ctr++, ring.next()) {
        const uint32_t slot = ring.slot;
        if (ctr >= C::RS && !mbar_wait(&raw_empty[slot], ring.phase ^ 1, ab)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          // half h: pair mode, 64-row tile `tile` of mats[mat + h]; else tile 2 tile + h of mats[mat]
          const GemmMat& m0 = a.mats[it.mat];
          const GemmMat& m1 = a.mats[a.pair ? it.mat + 1 : it.mat];
          const uint32_t t0 = a.pair ? it.tile : 2 * it.tile, t1 = a.pair ? it.tile : 2 * it.tile + 1;
          const bool h1 = t1 < m1.tiles;
          mbar_expect(&raw_full[slot], (h1 ? 2 : 1) * half_bytes);
          uint8_t* dst = raw + slot * raw_bytes;
          bulk_copy(dst, m0.w + it.e * m0.expert_stride + t0 * m0.tile_bytes + b * half_bytes, half_bytes,
                    &raw_full[slot]);
          if (h1)
            bulk_copy(dst + half_bytes, m1.w + it.e * m1.expert_stride + t1 * m1.tile_bytes + b * half_bytes,
                      half_bytes, &raw_full[slot]);
        }
      }
    }
    if (lane == 0)  // drain: the copies of the last stages issued
      for (uint32_t k = ctr > C::RS ? ctr - C::RS : 0; k < ctr; k++) mbar_drain(&raw_full[k % C::RS], (k / C::RS) & 1);
  } else if (warp == 2) {
    // ---- B planes of each stage's K steps: two bulk copies (hi, lo) per K step ----
    if (lane == 0) {
      uint32_t ctr = 0;
      Ring ring(SS);
      bool ok = true;
      ItemDesc nx{};
      if (blockIdx.x < nitems) nx = load_item(a, g0, blockIdx.x);
      for (uint32_t i = blockIdx.x; i < nitems && ok; i += gridDim.x) {
        const ItemDesc it = nx;
        if (i + gridDim.x < nitems) nx = load_item(a, g0, i + gridDim.x);
        const uint8_t* gimg = a.img + (uint64_t)it.imgoff * img_row;
        for (uint32_t s0 = 0; s0 < S; s0 += C::KS, ctr++, ring.next()) {
          const uint32_t slot = ring.slot;
          if (ctr >= SS && !mbar_wait(&st_empty[slot], ring.phase ^ 1, ab)) {
            ok = false;
            break;
          }
          uint32_t bytes = 0;
#pragma unroll
          for (uint32_t j = 0; j < C::KS; j++) bytes += 2 * it.N * kcs_of(s0 + j, a.img_hasmin) * 16;
          mbar_expect(&st_full[slot], bytes);
#pragma unroll
          for (uint32_t j = 0; j < C::KS; j++) {
            const uint32_t s = s0 + j, kcs = kcs_of(s, a.img_hasmin), plane = it.N * kcs * 16;
            const uint8_t* src = gimg + (uint64_t)it.nimg * 32 * kc_before(s, a.img_hasmin) + (it.n0 / 8) * kcs * 128;
            uint8_t* dst = stg + slot * stage_bytes + a_part + j * b_sub;
            bulk_copy(dst, src, plane, &st_full[slot]);
            bulk_copy(dst + plane, src + (uint64_t)it.nimg * kcs * 16, plane, &st_full[slot]);
          }
        }
      }
      for (uint32_t k = ctr > SS ? ctr - SS : 0; k < ctr; k++) mbar_drain(&st_full[k % SS], (k / SS) & 1);
    }
  } else if (warp == 1) {
    // ---- MMA issue (one thread) ----
    if (lane == 0) {
      uint32_t items = 0;
      Ring sr(SS);
      bool ok = true;
      uint64_t* last = nullptr;
      uint32_t last_par = 0;
      const uint32_t NP = a.NP;
      // descriptors of stage 0 (A; B of each K step per chunk count): slot k is k * stage_bytes further
      const unsigned long long ad0 = sdesc(smem_u32(stg), 128, C::kcsA * 128);
      const unsigned long long bd8 = sdesc(smem_u32(stg + a_part), 128, 8 * 128),
                               bd10 = sdesc(smem_u32(stg + a_part), 128, 10 * 128);
      ItemDesc nx{};
      if (blockIdx.x < nitems) nx = load_item(a, g0, blockIdx.x);
      for (uint32_t i = blockIdx.x; i < nitems && ok; i += gridDim.x, items++) {
        const ItemDesc it = nx;
        if (i + gridDim.x < nitems) nx = load_item(a, g0, i + gridDim.x);
        // f32 accumulator, f16 A and B, both K-major, M = 128, N = 2 x the pass's vectors: a B K step
        // holds the hi plane then the lo plane of the vectors, so one MMA multiplies A by both (columns
        // 0 .. N-1: hi, N .. 2N-1: lo; the epilogue adds the halves)
        const uint32_t idesc = (1u << 4) | (((2 * it.N) >> 3) << 17) | ((128u >> 4) << 24);
        for (uint32_t s0 = 0; s0 < S; s0 += C::KS, sr.next()) {
          if (!mbar_wait(&st_full[sr.slot], sr.phase, ab)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const unsigned long long so = (unsigned long long)(sr.slot * stage_bytes) >> 4;
#pragma unroll
          for (uint32_t j = 0; j < C::KS; j++) {
            const uint32_t s = s0 + j, sb = s >> 2;
            // K step j's A chunks start 8 j chunks into the row group; a K = 16 step is +256 bytes (16 units)
            const unsigned long long ad = ad0 + so + j * 64;
            const unsigned long long bd = (kcs_of(s, a.img_hasmin) == 10 ? bd10 : bd8) + so + (j * b_sub >> 4);
            const uint32_t dcol = tmem + sb * 2 * NP;
            if ((s & 3) == 0) mma_first(dcol, ad, bd, idesc);
            else mma_acc(dcol, ad, bd, idesc);
            mma_acc(dcol, ad + 16, bd + 16, idesc);
            mma_acc(dcol, ad + 32, bd + 32, idesc);
            mma_acc(dcol, ad + 48, bd + 48, idesc);
            if (AK == Q6_K) {  // the lo plane of A, 128 x 8 chunks further
              const unsigned long long al = ad + (128 * C::kcsA * 16 >> 4);
              mma_acc(dcol, al, bd, idesc);
              mma_acc(dcol, al + 16, bd + 16, idesc);
              mma_acc(dcol, al + 32, bd + 32, idesc);
              mma_acc(dcol, al + 48, bd + 48, idesc);
            }
            if (hasminA && (s & 3) == 3) {  // the min term of super-block sb: A chunks 8 KS, 8 KS + 1; B 8, 9
              const unsigned long long am = ad0 + so + 8 * C::KS * 8;
              if (sb == 0) mma_first(tmem + nsb * 2 * NP, am, bd + 64, idesc);
              else mma_acc(tmem + nsb * 2 * NP, am, bd + 64, idesc);
            }
          }
          mma_commit(&st_empty[sr.slot]);
          last = &st_empty[sr.slot];
          last_par = sr.phase;
        }
        if (!ok) break;
        mma_commit(&acc_full);
        last = &acc_full;
        last_par = items & 1;
      }
      if (last) mbar_drain(last, last_par);  // every MMA issued has completed
    }
  } else if (warp >= kProdWarp0) {
    // ---- A producers and epilogue: row r, half `part` of each K step ----
    const uint32_t pt = tid - kProdWarp0 * 32, part = pt >> 7, r = pt & 127;
    const uint32_t quarter = (warp - kProdWarp0) & 3;  // TMEM lanes 32 * quarter ..
    float* dme = dsm + part * nsb * 128;
    uint32_t sctr = 0, items = 0, pphase = 0;
    Ring rr(C::RS), sr(SS);
    bool ok = true;
    for (uint32_t i = blockIdx.x; i < nitems && ok; i += gridDim.x, items++) {
      const Item it = decode_item(a, g0, i);
      const QgGroup& g = group_at(a, it.g);
      uint32_t mi, row;
      const bool valid = tile_row(a, g.mat, it.tile, r, &mi, &row);
      const float smin = hasminA ? a.smin[mi] : 1.f;
      float* hsv = hsm + (items & 1) * a.NP;
      uint32_t* ysv = ysm + (items & 1) * a.NP;
      // the scale and output row of vector pt of the pass: loads in flight during the item
      float hs_pt = 1.f;
      uint32_t y_pt = 0;
      if (pt < it.N) {
        const uint32_t n = it.n0 + pt;
        if (a.hs && n < g.cnt) hs_pt = a.hs[g.hsmap ? g.hsmap[n] : n];
        if (EPI == 0 && n < g.cnt) y_pt = g.ymap ? g.ymap[n] : n;
      }
      for (uint32_t b = 0; b < nsb && ok; b++, rr.next()) {
        const uint32_t rs = rr.slot;
        if (!mbar_wait(&raw_full[rs], rr.phase, ab)) {
          ok = false;
          break;
        }
        const uint8_t* rw = raw + rs * raw_bytes + (r >> 6) * half_bytes + (r & 63) * C::blk;
        // per super-block: the row's block header and all of this thread's bytes of the 4 K steps
        float d = 0.f, dmin = 0.f;
        uint32_t sc03 = 0, sc47 = 0, mnp = 0;  // Q4_K: 6-bit scales of sub-blocks 0-3, 4-7; mins of 4 part..
        uint4 qv[4];                          // Q4_K: qs bytes 32 c + 16 part.  Q6_K: ql, ql + 16, qh, qh + 16
        if (AK == Q4_K) {
          uint4 h = make_uint4(0, 0, 0, 0);
          if (valid) {
            h = ld16<true>(rw);
#pragma unroll
            for (int c = 0; c < 4; c++) qv[c] = ld16<true>(rw + 16 + 32 * c + 16 * part);
          } else {
#pragma unroll
            for (int c = 0; c < 4; c++) qv[c] = make_uint4(0, 0, 0, 0);
          }
          d = h2f_bits(h.x);
          dmin = h2f_bits(h.x >> 16);
          // quant.rs get_scale_min_k4, four sub-blocks per word: bytes s[0..11] = h.y, h.z, h.w
          sc03 = h.y & 0x3f3f3f3fu;
          sc47 = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
          mnp = part == 0 ? (h.z & 0x3f3f3f3fu) : (((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u));
        } else {
          if (valid) {
            d = __half2float(*reinterpret_cast<const __half*>(raw + rs * raw_bytes + (r >> 6) * half_bytes + 64 * 208 +
                                                              (r & 63) * 2));
          }
        }
        dme[b * 128 + r] = d;
#pragma unroll
        for (uint32_t c = 0; c < 4; c++) {
          const uint32_t j = c % C::KS;  // K step within the stage
          if (j == 0 && sctr >= SS && !mbar_wait(&st_empty[sr.slot], sr.phase ^ 1, ab)) {
            ok = false;
            break;
          }
          uint8_t* Arow = stg + sr.slot * stage_bytes + (r >> 3) * (C::kcsA * 128) + (r & 7) * 16;
          uint8_t* A = Arow + j * 8 * 128;
          if (AK == Q4_K) {
            // low nibbles = sub-block 2c (weight sc * q), high nibbles = 2c + 1: 1024 + 16 q as fp16, times
            // sc / 16, minus 64 sc (exact: the results are integers below 2^10)
            const uint32_t scw = c < 2 ? sc03 : sc47, sh = 16 * (c & 1);
            const __half2 one024 = __float2half2_rn(1024.f);
            const __half2 s0 = __hsub2(u2h(prmt(scw >> sh, 0x64646464u, 0x4040u)), one024);  // (sc, sc)
            const __half2 s1 = __hsub2(u2h(prmt(scw >> sh, 0x64646464u, 0x4141u)), one024);
            const __half2 c0 = __hmul2(s0, __float2half2_rn(-1024.f));
            const __half2 s1q = __hmul2(s1, __float2half2_rn(0.0625f)), c1 = __hmul2(s1, __float2half2_rn(-64.f));
            const uint32_t w[4] = {qv[c].x, qv[c].y, qv[c].z, qv[c].w};
            uint32_t lo[8], hi[8];
#pragma unroll
            for (int k = 0; k < 4; k++) {
              const uint32_t t0 = prmt(w[k], 0x64646464u, 0x4140u), t1 = prmt(w[k], 0x64646464u, 0x4342u);
              lo[2 * k] = h2u(__hfma2(u2h(t0 & 0xff0fff0fu), s0, c0));
              lo[2 * k + 1] = h2u(__hfma2(u2h(t1 & 0xff0fff0fu), s0, c0));
              hi[2 * k] = h2u(__hfma2(u2h(t0 & 0xfff0fff0u), s1q, c1));
              hi[2 * k + 1] = h2u(__hfma2(u2h(t1 & 0xfff0fff0u), s1q, c1));
            }
            *reinterpret_cast<uint4*>(A + (2 * part) * 128) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            *reinterpret_cast<uint4*>(A + (2 * part + 1) * 128) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
            *reinterpret_cast<uint4*>(A + (4 + 2 * part) * 128) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(A + (5 + 2 * part) * 128) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
            if (c == 3) {  // min block: dmin * mn_j * s_min for sub-blocks j = 4 part .. + 3, hi | lo
              const float ds = dmin * smin;
              float v[4];
#pragma unroll
              for (int k = 0; k < 4; k++) v[k] = ds * (float)((mnp >> (8 * k)) & 0xffu);
              uint32_t h0, l0, h1, l1;
              split2(v[0], v[1], &h0, &l0);
              split2(v[2], v[3], &h1, &l1);
              *reinterpret_cast<uint2*>(Arow + 8 * C::KS * 128 + 8 * part) = make_uint2(h0, h1);
              *reinterpret_cast<uint2*>(Arow + (8 * C::KS + 1) * 128 + 8 * part) = make_uint2(l0, l1);
            }
          } else {
            // K step c of the super-block: half nh = c / 2, quarter qa = 2 (c % 2) + part (32 weights)
            const uint32_t nh = c >> 1, qa = 2 * (c & 1) + part;
            if ((c & 1) == 0) {  // ql and qh bytes shared by K steps c and c + 1
              if (valid) {
                const uint8_t* ql = rw + 64 * nh + 32 * part;
                qv[0] = ld16<true>(ql);
                qv[1] = ld16<true>(ql + 16);
                qv[2] = ld16<true>(rw + 128 + 32 * nh);
                qv[3] = ld16<true>(rw + 128 + 32 * nh + 16);
              } else {
#pragma unroll
                for (int q = 0; q < 4; q++) qv[q] = make_uint4(0, 0, 0, 0);
              }
            }
            uint32_t scb = 0;
            if (valid) scb = *reinterpret_cast<const unsigned short*>(rw + 192 + 8 * nh + 2 * qa);
            const uint32_t nsh = 4 * (c & 1), hsh = 2 * qa;
            const uint32_t lw[8] = {qv[0].x, qv[0].y, qv[0].z, qv[0].w, qv[1].x, qv[1].y, qv[1].z, qv[1].w};
            const uint32_t hw[8] = {qv[2].x, qv[2].y, qv[2].z, qv[2].w, qv[3].x, qv[3].y, qv[3].z, qv[3].w};
            const __half2 m1056 = __float2half2_rn(-1056.f);
#pragma unroll
            for (int half16 = 0; half16 < 2; half16++) {  // weights 16 half16 .. + 15 share scale byte half16
              const __half2 sv = __float2half2_rn((float)(int8_t)((scb >> (8 * half16)) & 0xff));
              uint32_t ahi[8], alo[8];
#pragma unroll
              for (int k = 0; k < 4; k++) {
                const uint32_t wl = lw[4 * half16 + k], wh = hw[4 * half16 + k];
                const uint32_t hq = hsh <= 4 ? (wh << (4 - hsh)) : (wh >> (hsh - 4));
                const uint32_t q = ((wl >> nsh) & 0x0f0f0f0fu) | (hq & 0x30303030u);
                const __half2 u0 = __hadd2(u2h(prmt(q, 0x64646464u, 0x4140u)), m1056);
                const __half2 u1 = __hadd2(u2h(prmt(q, 0x64646464u, 0x4342u)), m1056);
                const __half2 p0 = __hmul2(u0, sv), p1 = __hmul2(u1, sv);
                ahi[2 * k] = h2u(p0);
                ahi[2 * k + 1] = h2u(p1);
                alo[2 * k] = h2u(__hfma2(u0, sv, __hneg2(p0)));
                alo[2 * k + 1] = h2u(__hfma2(u1, sv, __hneg2(p1)));
              }
              const uint32_t ch = 4 * part + 2 * half16;  // chunks of this thread's 16 weights
              uint8_t* Al = A + 128 * C::kcsA * 16;
              *reinterpret_cast<uint4*>(A + ch * 128) = make_uint4(ahi[0], ahi[1], ahi[2], ahi[3]);
              *reinterpret_cast<uint4*>(A + (ch + 1) * 128) = make_uint4(ahi[4], ahi[5], ahi[6], ahi[7]);
              *reinterpret_cast<uint4*>(Al + ch * 128) = make_uint4(alo[0], alo[1], alo[2], alo[3]);
              *reinterpret_cast<uint4*>(Al + (ch + 1) * 128) = make_uint4(alo[4], alo[5], alo[6], alo[7]);
            }
          }
          if (j == C::KS - 1) {  // the stage's A part is written
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&st_full[sr.slot]);
            sctr++;
            sr.next();
          }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);
      }
      if (!ok) break;
      // ---- epilogue: y[n][row] = (sum_b d_b acc_b + kmin acc_min) / hs_n ----
      if (!mbar_wait(&acc_full, items & 1, ab)) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (pt < it.N) {
        hsv[pt] = 1.f / hs_pt;
        ysv[pt] = y_pt;
      }
      if (!prod_sync(&psync, &pphase, ab)) {  // hsv, ysv of this item are written
        ok = false;
        break;
      }
      const uint32_t cols = it.N / 2, c0 = part * cols;  // (N a multiple of 8)
      const float kmin = hasminA ? 32.f / smin : 0.f;
      float* E = reinterpret_cast<float*>(stg);  // EPI 1: [128][NP + 1] (the stages are consumed)
      for (uint32_t cc = 0; cc < cols; cc += 4) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t taddr = tmem + ((quarter * 32) << 16) + c0 + cc, nacc = nsb + (hasminA ? 1 : 0);
        for (uint32_t b0 = 0; b0 < nacc; b0 += 4) {  // up to 4 accumulators (hi and lo halves) per wait
          uint32_t v[4][8];
#pragma unroll
          for (uint32_t q = 0; q < 4; q++)
            if (b0 + q < nacc) {
              const uint32_t t = taddr + (b0 + q) * 2 * a.NP;
              asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(v[q][0]), "=r"(v[q][1]), "=r"(v[q][2]), "=r"(v[q][3])
                           : "r"(t));
              asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(v[q][4]), "=r"(v[q][5]), "=r"(v[q][6]), "=r"(v[q][7])
                           : "r"(t + it.N));
            }
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (uint32_t q = 0; q < 4; q++)
            if (b0 + q < nacc) {
              const float f = b0 + q < nsb ? dme[(b0 + q) * 128 + r] : kmin;
#pragma unroll
              for (int k = 0; k < 4; k++)
                acc[k] = fmaf(f, __uint_as_float(v[q][k]) + __uint_as_float(v[q][4 + k]), acc[k]);
            }
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const uint32_t n = c0 + cc + k;
          const float out = acc[k] * hsv[n];
          if (EPI == 0) {
            if (valid && n < it.nn) {
              const uint64_t at = (uint64_t)ysv[n] * g.ystride + row;
              g.y[at] = g.add ? __fadd_rn(g.add[at], out) : out;
            }
          } else {
            E[r * (a.NP + 1) + n] = out;
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      if (EPI == 1) {
        // SwiGLU of gate row j (tile rows 0-63) and up row j (64-127), into the next GEMM's image:
        // K step `tile`, chunk j / 8, vector n (model.rs:259-274: g / (1 + exp(-g)) * u)
        if (!prod_sync(&psync, &pphase, ab)) {
          ok = false;
          break;
        }
        const uint32_t h2 = a.img2_hasmin, row2 = 32 * kc_before(a.K2 / 64, h2), kcs2 = kcs_of(it.tile, h2);
        uint8_t* gimg2 = a.img2 + (uint64_t)g.imgoff * row2 + (uint64_t)g.nimg * 32 * kc_before(it.tile, h2);
        // with min chunks: this tile's two sub-block sums go to halves 2 (tile % 4) + {0, 1} of the
        // min chunks of its super-block's last K step
        uint8_t* gmin = a.img2 + (uint64_t)g.imgoff * row2 + (uint64_t)g.nimg * 32 * kc_before(it.tile | 3, h2);
        for (uint32_t q = pt; q < it.N * 8; q += kProd) {
          const uint32_t n = q >> 3, jc = q & 7;
          float v[8];
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const uint32_t j = jc * 8 + k;
            const float gg = E[j * (a.NP + 1) + n], uu = E[(64 + j) * (a.NP + 1) + n];
            const bool ok_j = n < it.nn && it.tile * 64 + j < a.mats[g.mat].rows;  // (gate rows)
            const float act = ok_j ? __fmul_rn(__fdiv_rn(gg, __fadd_rn(1.f, expf(-gg))), uu) : 0.f;
            if (!(fabsf(act) < 65504.f)) atomicOr(a.err, 4u);  // outside the fp16 range of the image
            v[k] = act;
          }
          uint32_t h[4], l[4];
#pragma unroll
          for (int k = 0; k < 4; k++) split2(v[2 * k], v[2 * k + 1], &h[k], &l[k]);
          const uint32_t ng = it.n0 + n;
          uint8_t* dst = gimg2 + (ng >> 3) * (kcs2 * 128) + jc * 128 + (ng & 7) * 16;
          *reinterpret_cast<uint4*>(dst) = make_uint4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<uint4*>(dst + (uint64_t)g.nimg * kcs2 * 16) = make_uint4(l[0], l[1], l[2], l[3]);
          if (h2) {  // sums of 32 outputs: the 4 lanes jc = 4 sb .. 4 sb + 3 of vector n
            float xs = 0.f;
#pragma unroll
            for (int k = 0; k < 8; k++) xs += v[k];
            xs += __shfl_xor_sync(0xffffffffu, xs, 1);
            xs += __shfl_xor_sync(0xffffffffu, xs, 2);
            if ((jc & 3) == 0) {
              const __half2 hh = __floats2half2_rn(-xs * 0.03125f, 0.f);
              const float back = __low2float(hh);
              const __half hl = __float2half_rn(-xs * 0.03125f - back);
              const uint32_t pos = 2 * (it.tile & 3) + (jc >> 2);  // half index in the min chunks
              uint8_t* m = gmin + (ng >> 3) * (10 * 128) + (ng & 7) * 16 + 2 * pos;
              uint8_t* ml = m + (uint64_t)g.nimg * 10 * 16;
              *reinterpret_cast<__half*>(m + 8 * 128) = __low2half(hh);
              *reinterpret_cast<__half*>(m + 9 * 128) = __low2half(hh);
              *reinterpret_cast<__half*>(ml + 8 * 128) = hl;
              *reinterpret_cast<__half*>(ml + 9 * 128) = __float2half_rn(0.f);
            }
          }
        }
        if (!prod_sync(&psync, &pphase, ab)) {  // E (the A stages) is free again
          ok = false;
          break;
        }
      }
    }
  }
  if (abort_flag && tid == 0) atomicOr(a.err, 2u);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
}

// ---- B image -----------------------------------------------------------------------------------
// Image row i: the vector of source row src (x[src * xstride ..], K floats), optionally RMS-normalized
// with weight w (ops.rs:3-15: x_i * (s * w_i)), times hs (a power of two: given per source row, or
// chosen here from the row's largest |value| and written to hs_out[i]), as fp16 hi + lo.  Rows
// without a source are zeros.  With min chunks, the last K step of each super-block carries the
// sub-block sums: chunk 8 = chunk 9 = hi(-sum * 2^-5) in the hi plane, chunk 8 = lo(.), chunk 9 = 0
// in the lo plane.
__global__ void __launch_bounds__(256) k_qg_image(QgImageArgs a) {
  __shared__ float red[32];
  const uint32_t i = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  uint32_t src, imgoff, nimg;
  if (a.rows) {
    if (i >= *a.nrows) return;
    const uint4 d = a.rows[i];
    src = d.x;
    imgoff = d.y;
    nimg = d.z;
  } else {
    if (i >= ((a.T + 15) & ~15u)) return;
    src = i < a.T ? (a.src ? a.src[i] : i) : kNone;
    imgoff = 0;
    nimg = (a.T + 15) & ~15u;
  }
  const uint32_t K = a.K, S = K / 64, n = i - imgoff, chunks = K / 8;
  const uint32_t row_bytes = 32 * kc_before(S, a.hasmin);
  uint8_t* base = a.img + (uint64_t)imgoff * row_bytes;
  constexpr uint32_t kMaxPer = 4;  // chunks per thread (K <= 8192)
  float v[kMaxPer][8];
  const float* x = src != kNone ? a.x + (uint64_t)src * a.xstride : nullptr;
  const bool x16 = x && (reinterpret_cast<uintptr_t>(x) & 15) == 0;  // 8 floats as two 16-byte loads
#pragma unroll
  for (uint32_t p = 0; p < kMaxPer; p++) {
    const uint32_t t = tid + 256 * p;
    if (x16 && t < chunks) {
      const float4 u0 = reinterpret_cast<const float4*>(x)[2 * t], u1 = reinterpret_cast<const float4*>(x)[2 * t + 1];
      v[p][0] = u0.x, v[p][1] = u0.y, v[p][2] = u0.z, v[p][3] = u0.w;
      v[p][4] = u1.x, v[p][5] = u1.y, v[p][6] = u1.z, v[p][7] = u1.w;
    } else {
#pragma unroll
      for (int k = 0; k < 8; k++) v[p][k] = (x && t < chunks) ? x[8 * t + k] : 0.f;
    }
  }
  if (a.w) {  // RMSNorm
    float ss = 0.f;
#pragma unroll
    for (uint32_t p = 0; p < kMaxPer; p++)
#pragma unroll
      for (int k = 0; k < 8; k++) ss = fmaf(v[p][k], v[p][k], ss);
    ss = block_sum(ss, red);
    const float s = 1.0f / sqrtf(ss / (float)K + a.eps);
    const bool w16 = (reinterpret_cast<uintptr_t>(a.w) & 15) == 0;
#pragma unroll
    for (uint32_t p = 0; p < kMaxPer; p++) {
      const uint32_t t = tid + 256 * p;
      float w[8];
      if (w16 && t < chunks) {
        const float4 u0 = reinterpret_cast<const float4*>(a.w)[2 * t], u1 = reinterpret_cast<const float4*>(a.w)[2 * t + 1];
        w[0] = u0.x, w[1] = u0.y, w[2] = u0.z, w[3] = u0.w, w[4] = u1.x, w[5] = u1.y, w[6] = u1.z, w[7] = u1.w;
      } else {
#pragma unroll
        for (int k = 0; k < 8; k++) w[k] = t < chunks ? a.w[8 * t + k] : 0.f;
      }
#pragma unroll
      for (int k = 0; k < 8; k++) v[p][k] = t < chunks ? __fmul_rn(v[p][k], __fmul_rn(s, w[k])) : 0.f;
    }
  }
  float hs;
  if (a.hs_in) {
    hs = src != kNone ? a.hs_in[src] : 1.f;
  } else {
    float mx = 0.f;
#pragma unroll
    for (uint32_t p = 0; p < kMaxPer; p++)
#pragma unroll
      for (int k = 0; k < 8; k++) mx = fmaxf(mx, fabsf(v[p][k]));
    mx = warp_max(mx);
    __syncthreads();
    if (lane == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = 0.f;
    for (uint32_t w = 0; w < 8; w++) mx = fmaxf(mx, red[w]);
    hs = qg_pow2_scale(mx);
    if (tid == 0 && a.hs_out) a.hs_out[i] = hs;
  }
#pragma unroll
  for (uint32_t p = 0; p < kMaxPer; p++) {
    const uint32_t t = tid + 256 * p;
    if (256 * p >= chunks) break;  // (block-uniform)
    float xs = 0.f;
    uint32_t h[4] = {0, 0, 0, 0}, l[4] = {0, 0, 0, 0};
    if (t < chunks) {
#pragma unroll
      for (int k = 0; k < 8; k++) {
        v[p][k] *= hs;
        xs += v[p][k];
      }
#pragma unroll
      for (int k = 0; k < 4; k++) split2(v[p][2 * k], v[p][2 * k + 1], &h[k], &l[k]);
      const uint32_t s = t >> 3, kc = t & 7, kcs = kcs_of(s, a.hasmin);
      uint8_t* dst = base + (uint64_t)nimg * 32 * kc_before(s, a.hasmin) + (n >> 3) * kcs * 128 + kc * 128 + (n & 7) * 16;
      *reinterpret_cast<uint4*>(dst) = make_uint4(h[0], h[1], h[2], h[3]);
      *reinterpret_cast<uint4*>(dst + (uint64_t)nimg * kcs * 16) = make_uint4(l[0], l[1], l[2], l[3]);
    }
    if (a.hasmin) {  // sub-block sums: 4 chunks per sub-block, a warp per super-block (32 chunks)
      xs += __shfl_xor_sync(0xffffffffu, xs, 1);
      xs += __shfl_xor_sync(0xffffffffu, xs, 2);
      float sj[8];
#pragma unroll
      for (int j = 0; j < 8; j++) sj[j] = -__shfl_sync(0xffffffffu, xs, 4 * j) * 0.03125f;
      if (lane == 0 && t < chunks) {
        uint32_t hh[4], ll[4];
#pragma unroll
        for (int k = 0; k < 4; k++) split2(sj[2 * k], sj[2 * k + 1], &hh[k], &ll[k]);
        const uint32_t s = (t >> 3) | 3, kcs = 10;  // the super-block's last K step
        uint8_t* dst = base + (uint64_t)nimg * 32 * kc_before(s, 1) + (n >> 3) * kcs * 128 + (n & 7) * 16;
        uint8_t* dl = dst + (uint64_t)nimg * kcs * 16;
        *reinterpret_cast<uint4*>(dst + 8 * 128) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
        *reinterpret_cast<uint4*>(dst + 9 * 128) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
        *reinterpret_cast<uint4*>(dl + 8 * 128) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
        *reinterpret_cast<uint4*>(dl + 9 * 128) = make_uint4(0, 0, 0, 0);
      }
    }
  }
}

// Largest |dmin| over a Q4_K matrix (atomic max of the float bits).
__global__ void k_qg_dmin(MatDesc m, uint32_t experts, uint32_t* out) {
  const uint32_t blocks = m.cols / 256;
  const uint64_t n = (uint64_t)experts * m.rows * blocks;
  float mx = 0.f;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = (uint32_t)(i / ((uint64_t)m.rows * blocks)), rem = (uint32_t)(i % ((uint64_t)m.rows * blocks));
    const uint8_t* b = row_ptr(m, expert_base(m, e), rem / blocks) + (rem % blocks) * 144;
    const float dmin = fabsf(h2f_bits(b[2] | (b[3] << 8)));
    if (isfinite(dmin)) mx = fmaxf(mx, dmin);
  }
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(mx));
}

// One thread per (expert, 64-row tile, super-block, row): the row's block (and d value) to the GEMM layout.
__global__ void k_qg_relayout(MatDesc m, uint32_t experts, GemmMat g) {
  const uint32_t nsb = m.cols / 256, blk = m.kind == Q4_K ? 144 : 208;
  const uint64_t total = (uint64_t)experts * g.tiles * nsb * 64;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t rr = (uint32_t)(i & 63);
    uint64_t q = i >> 6;
    const uint32_t b = (uint32_t)(q % nsb);
    q /= nsb;
    const uint32_t t = (uint32_t)(q % g.tiles), e = (uint32_t)(q / g.tiles), row = t * 64 + rr;
    uint8_t* blockp = const_cast<uint8_t*>(g.w) + e * g.expert_stride + t * g.tile_bytes + b * g.blockb;
    uint4* dst = reinterpret_cast<uint4*>(blockp + rr * blk);
    if (row < m.rows) {
      const uint8_t* base = expert_base(m, e);
      const uint4* src = reinterpret_cast<const uint4*>(row_ptr(m, base, row) + b * blk);
      for (uint32_t k = 0; k < blk / 16; k++) dst[k] = src[k];
      if (m.kind == Q6_K) reinterpret_cast<__half*>(blockp + 64 * 208)[rr] = drow_ptr(m, base, row)[b];
    } else {
      for (uint32_t k = 0; k < blk / 16; k++) dst[k] = make_uint4(0, 0, 0, 0);
      if (m.kind == Q6_K) reinterpret_cast<__half*>(blockp + 64 * 208)[rr] = __float2half_rn(0.f);
    }
  }
}

}  // namespace

void launch_qg_relayout(const MatDesc& src, uint32_t experts, const GemmMat& dst, cudaStream_t s) {
  k_qg_relayout<<<148 * 8, 256, 0, s>>>(src, experts, dst);
}

const char* qgemm_supported(uint32_t kind, uint32_t cols) {
  if (kind != Q4_K && kind != Q6_K) return "the tensor-core GEMM takes Q4_K and Q6_K rows";
  if (cols % 256) return "the tensor-core GEMM needs a multiple of 256 columns";
  const uint32_t acc = cols / 256 + (kind == Q4_K ? 1 : 0);
  if (acc > 32 || cols > 8192) return "the tensor-core GEMM takes at most 8192 columns";
  if (kind == Q6_K && cols > 4096) return "the tensor-core GEMM takes at most 4096 columns of Q6_K rows";
  return nullptr;
}

uint64_t qg_image_row_bytes(uint32_t cols, bool hasmin) {
  const uint64_t S = cols / 64;
  return 32 * (8 * S + (hasmin ? 2 * (S / 4) : 0));
}

// Shared memory besides the stages, and one stage (the A operand of KS K steps and their B planes).
static size_t qgemm_fixed(uint32_t kind, uint32_t cols, uint32_t np) {
  const uint32_t nsb = cols / 256;  // (+ 1 KB: the carve-up is aligned to 1 KB)
  const size_t f = kind == Q4_K ? Cfg<Q4_K>::RS * 128 * 144 : Cfg<Q6_K>::RS * 128 * 210;
  return f + 2 * nsb * 128 * 4 + 2 * np * 8 + 1024;
}
static size_t qgemm_stage(uint32_t kind, uint32_t np, bool img_hasmin) {
  const size_t b = 2 * np * (img_hasmin ? 10 : 8) * 16;
  return kind == Q4_K ? a_stage_bytes<Q4_K>() + Cfg<Q4_K>::KS * b : a_stage_bytes<Q6_K>() + Cfg<Q6_K>::KS * b;
}

size_t qgemm_smem(uint32_t kind, uint32_t cols, uint32_t np, uint32_t ss, bool img_hasmin) {
  return qgemm_fixed(kind, cols, np) + ss * qgemm_stage(kind, np, img_hasmin);
}

static size_t g_qgemm_cap = 0;  // dynamic shared memory every GEMM kernel may use (set by qgemm_prepare)

template <class F>
static cudaError_t qgemm_attr(F* f, int optin, size_t* cap) {
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, f);
  if (e != cudaSuccess) return e;
  const int c = optin - (int)fa.sharedSizeBytes;
  if (c <= 0) return cudaErrorInvalidValue;
  e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, c);
  if ((size_t)c < *cap) *cap = (size_t)c;
  return e;
}

cudaError_t qgemm_prepare() {
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  size_t cap = ~(size_t)0;
  if (e == cudaSuccess) e = qgemm_attr(k_qgemm<Q4_K, 0>, optin, &cap);
  if (e == cudaSuccess) e = qgemm_attr(k_qgemm<Q4_K, 1>, optin, &cap);
  if (e == cudaSuccess) e = qgemm_attr(k_qgemm<Q6_K, 0>, optin, &cap);
  if (e == cudaSuccess) e = qgemm_attr(k_qgemm<Q6_K, 1>, optin, &cap);
  if (e == cudaSuccess) g_qgemm_cap = cap;
  return e;
}

size_t qgemm_smem_cap() { return g_qgemm_cap; }

// Vectors per pass (NP) and stages (SS).  NP: as large as the TMEM accumulators allow (one per
// super-block and the Q4_K min accumulator, 2 NP columns each: at most 512), up to 64, a multiple of
// 8; lowered until 3 stages fit (up to 8).
const char* qgemm_shape(uint32_t kind, uint32_t cols, bool img_hasmin, uint32_t* np, uint32_t* ss) {
  if (const char* why = qgemm_supported(kind, cols)) return why;
  const uint32_t acc = cols / 256 + (kind == Q4_K ? 1 : 0);
  uint32_t n = 512 / (2 * acc) / 8 * 8;  // (each accumulator: 2 n columns)
  n = n > 64 ? 64 : n;
  if (n < 8) return "the tensor-core GEMM takes at most 4096 columns of Q4_K rows";
  const size_t cap = g_qgemm_cap;
  for (;; n -= 8) {
    const size_t fixed = qgemm_fixed(kind, cols, n), st = qgemm_stage(kind, n, img_hasmin);
    const size_t k = fixed < cap ? (cap - fixed) / st : 0;
    if (k >= 3 || n == 8) {
      if (k < 2) return "the tensor-core GEMM needs more shared memory than this device has";
      *np = n;
      *ss = k > kMaxSS ? kMaxSS : (uint32_t)k;
      return nullptr;
    }
  }
}



void launch_qgemm(const QgArgs& a, uint32_t kind, bool swiglu, uint32_t grid, cudaStream_t s) {
  const size_t smem = qgemm_smem(kind, a.K, a.NP, a.SS, a.img_hasmin != 0);
  if (kind == Q4_K) {
    if (swiglu) k_qgemm<Q4_K, 1><<<grid, kThreads, smem, s>>>(a);
    else k_qgemm<Q4_K, 0><<<grid, kThreads, smem, s>>>(a);
  } else {
    if (swiglu) k_qgemm<Q6_K, 1><<<grid, kThreads, smem, s>>>(a);
    else k_qgemm<Q6_K, 0><<<grid, kThreads, smem, s>>>(a);
  }
}

void launch_qg_image(const QgImageArgs& a, uint32_t grid, cudaStream_t s) { k_qg_image<<<grid, 256, 0, s>>>(a); }

void launch_qg_dmin(const MatDesc& m, uint32_t experts, uint32_t* out, cudaStream_t s) {
  k_qg_dmin<<<296, 256, 0, s>>>(m, experts, out);
}

}  // namespace qc
