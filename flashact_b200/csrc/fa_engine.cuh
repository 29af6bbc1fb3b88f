// Model-independent engine of the denoise megakernels (sm_100a): warp / CTA helpers, the
// bounded grid barrier, stage tracing, and the three GEMM roles — weight producer (warp 0),
// tcgen05 MMA issuer (warp 1) and epilogue driver (warps 2-5). The roles are templates over a
// model-traits type that supplies the per-layer matrices (row counts, tensor maps, activation
// operand) and the fused epilogue; see pi05_kernel.cu and ma2_kernel.cu.
//
// Roles run as whole warps with uniform control flow; lane 0 alone issues TMA / tcgen05 /
// commit instructions. Every field a role needs is copied into registers at entry: the inline
// asm "memory" clobbers would otherwise force a reload through the generic Params / Ctx
// references after every TMA or mbarrier operation.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "fa_engine_types.cuh"
#include "fa_ptx.cuh"

namespace fa {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Named barriers: 1 = warps 1-5 (stage sequencing), 2 = warps 2-5 (epilogue group).
// barrier.sync (non-.aligned): warp 1 reaches it with lane 0 arriving after the other lanes.
__device__ __forceinline__ void sync_main() {
  __syncwarp();
  asm volatile("barrier.sync 1, 160;" ::: "memory");
}
__device__ __forceinline__ void sync_epi() {
  __syncwarp();
  asm volatile("barrier.sync 2, 128;" ::: "memory");
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Observation index of packed token n = b * T + t without an integer division: exact for
// n < 2^16 because (n + 0.5) / T stays at least 0.5 / T away from an integer.
__device__ __forceinline__ int tok_bi(float invT, int n) { return (int)(((float)n + 0.5f) * invT); }

// Stage tracing (diagnostics): g_trp points at this CTA's stamps for the current stage (null
// when the stage is not traced); g_t0 is the stage's start clock. Set by the barrier thread.
__shared__ unsigned long long* g_trp;
__shared__ unsigned long long g_t0;
// Compiled in only with -DFA_TRACE (diagnostic builds): the marks cost instruction-cache space
// in every stage.
__device__ __forceinline__ void trace_mark(int slot) {
#ifdef FA_TRACE
  unsigned long long* tr = g_trp;
  if (tr) tr[slot] = clock64() - g_t0;
#else
  (void)slot;
#endif
}

// gelu with the tanh approximation (src/pi05/mk6.cu:79-82).
// tanh by the hardware approximation (tanh.approx.f32, max relative error ~2^-11: below the
// bf16 rounding the result gets next).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(k0 * (x + 0.044715f * x * x * x)));
  return 0.5f * x * (1.0f + t);
}

// Grid barrier among warps 1-5 of every CTA. `gen` counts barriers passed by this launch; the
// counter only grows, so barrier k completes when it reaches (k+1) * gridDim.x. Bounded: on
// timeout (or when another CTA already failed) it raises *err and returns false.
// `overlap` runs on the epilogue warps (threads 64..191) between this CTA's arrival and the
// end of the wait: work that depends on no other CTA, hidden behind the barrier latency.
struct NoOverlap {
  __device__ void operator()() const {}
};
template <class P, class F = NoOverlap>
__device__ __forceinline__ bool grid_barrier(const P& p, uint32_t gen, unsigned long long* next_tr,
                                             const F& overlap = F()) {
  __shared__ int s_ok;
  sync_main();
  if (threadIdx.x >= 64) overlap();
  if (threadIdx.x == 32) {
    trace_mark(kTrBarArrive);
    int ok = 1;
    fence_proxy_async_global();
    // release-add: orders this CTA's earlier writes (made visible to this thread by the CTA
    // barrier above) before the arrival, without a separate full fence
    if (!(blockIdx.x == 0 && (int)gen == p.inject_barrier))
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
    const uint32_t target = (gen + 1) * gridDim.x;
    uint32_t i = 0;
    for (;; ++i) {
      uint32_t v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.bar) : "memory");
      if (v >= target) break;
      if (*(volatile int*)p.err) { ok = 0; break; }
      if (i > p.spin_limit) { atomicCAS(p.err, 0, KERR_BARRIER); ok = 0; break; }
      if (i > 64) __nanosleep(32);
    }
    fence_proxy_async_global();
    s_ok = ok;
#ifdef FA_TRACE
    g_t0 = clock64();
    g_trp = next_tr;
    if (next_tr) next_tr[kTrStart] = g_t0;
#else
    (void)next_tr;
#endif
  }
  sync_main();
  return s_ok != 0;
}

// Block-wide sum over the 128 epilogue threads.
__device__ __forceinline__ float epi_sum(float v, float* red) {
  const int e = threadIdx.x - 64;
  v = warp_sum(v);
  if ((e & 31) == 0) red[e >> 5] = v;
  sync_epi();
  float s = red[0] + red[1] + red[2] + red[3];
  sync_epi();
  return s;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The producer and MMA roles run as whole warps (uniform control flow, every lane waits on
// the same barriers) and only lane 0 issues TMA / tcgen05 / commit instructions.
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ bool leader() { return (threadIdx.x & 31) == 0; }
#define FA_ONE(stmt)      \
  do {                    \
    if (leader()) { stmt; } \
  } while (0)

// ------------------------------------------------------------------ CTA context
struct Bars {
  uint64_t wfull[kMaxRing], wempty[kMaxRing];
  uint64_t afull[kTmASlots], aempty[kTmASlots];  // FP8: TMEM A slot written / read by the MMAs
  uint64_t bfull, bempty;  // activation batch loaded / consumed
  uint64_t sfull[4];       // token-major GEMMs: activation K-chunk landed in staging slot 0..3
  uint64_t sempty[4];      // token-major GEMMs: the MMAs reading staging slot 0..3 have completed
  uint64_t acc_full[2], acc_empty[2];
  uint64_t q_full, k_full, v_full, kv_free, v_free, s_full, p_full, o_full, o_free, drain;
  uint64_t s_free, pv_done;  // whole-unit attention: S read by the softmax warps; P V done (P and V free)
  // MolmoAct2 whole-unit cross-attention (double-buffered S / P / O per 128-key chunk)
  uint64_t xq_full, xs_full[2], xs_free[2], xp_full[2], xo_full[2], xo_free[2];
};
struct Ctx {
  uint8_t* ring;  // ring_slots x (wg x 16 KB); FP8 streaming: ring_slots x (wg x 8 KB) of E4M3 codes
  uint8_t* work;  // activation atoms (GEMM) or Q | K/V | P (attention)
  Bars* bars;
  uint32_t tmem;
  int ring_slots;
  int tm_slots;             // token-major GEMMs: activation staging slots (2..4 chunks of 32 KB)
  int batoms;               // activation atoms that fit in the work area at once
  uint8_t* stage;           // 16 KB epilogue staging area (coalesced bf16 output writes)
  const GemmUnit* gu[kMaxMats];  // this CTA's units per matrix (shared-memory copy of the plan)
  int gcnt[kMaxMats];
  const AttnUnit* au;
  int acnt;
};

template <class P>
__device__ __forceinline__ int group_tiles(const P& p, int g) {
  const int tiles = p.NPAD / p.NTILE;
  const int rem = tiles - g * p.TG;
  return rem < p.TG ? rem : p.TG;
}

// ------------------------------------------------------------------ warp 0: weight producer
// Walks (step, layer, GEMM matrix, unit, token group, K-atom group) — the exact order the MMA
// lane consumes — and keeps the ring full. It never waits on activations.
template <class Model>
__device__ __forceinline__ void run_producer(const typename Model::Params& p, const Ctx& c) {
  // Every field is read once into registers: the inline-asm memory clobbers would otherwise
  // force a reload through the generic Params/Ctx references after each TMA / mbarrier op.
  // bs=1: every weight byte is read once per Euler step (evict first); several token groups
  // re-read each weight tile shortly after one another (keep it in L2)
  const uint64_t pol = p.ngroups > 1 ? policy_evict_normal() : policy_evict_first();
  const int R = c.ring_slots, nsteps = p.nsteps, L = p.L, wg = p.wg;
  // FP8 streaming: a slot holds the same K range in E4M3 (half the bytes); boxes are 128-byte
  // rows of 128 K-values, so the K coordinate counts pairs of bf16 atoms
  constexpr bool F8 = Model::kF8;
  const uint32_t slot_bytes = F8 ? (uint32_t)wg * kAtomBytes / 2 : (uint32_t)wg * kAtomBytes;
  uint8_t* const ring = c.ring;
  Bars* const bars = c.bars;
  int* const err = p.err;
  const CUtensorMap* const maps = p.maps;
  unsigned long long* const trace = p.trace;
  const int tstep = p.trace_step, tlayer = p.trace_layer;
  const GemmUnit* gul[Model::kMats];
  int gcnt[Model::kMats];
#pragma unroll
  for (int m = 0; m < Model::kMats; ++m) { gul[m] = c.gu[m]; gcnt[m] = c.gcnt[m]; }
  uint32_t it = 0;
  bool ok = true;
  // L2 prefetch of the weight stream, `ahead` layer-steps in front of the ring: HBM keeps
  // streaming while the dependent chain of a layer (attention, norms, barriers) runs, and the
  // GEMM stages then read their weights from L2. Each CTA prefetches exactly the rows and K
  // ranges of its own units, with all 32 lanes issuing line prefetches (prefetch.global.L2 goes
  // through the load/store path, so the TMA queue, which carries the ring and activation loads,
  // stays clear).
  const int ahead = p.l2_ahead, total_layers = nsteps * L;
  auto prefetch_layer = [&](int g) {
    if (g >= total_layers) return;
    const int lp = g % L;
#pragma unroll 1
    for (int m = 0; m < Model::kMats; ++m) {
      const int rows = Model::rows(m);
      const uint8_t* const wb = p.wraw[m];
      const size_t rb = (size_t)p.wrow_bytes[m];
      const int esz = F8 ? 1 : 2;
#pragma unroll 1
      for (int u = 0; u < gcnt[m]; ++u) {
        const GemmUnit gu = gul[m][u];
        if (gu.grp != 0) continue;  // token groups share a weight tile: prefetch it once
        const int nr = gu.half ? 64 : 128;
        const size_t r0 = (size_t)lp * rows + gu.mtile * 128 + (gu.half == 2 ? 64 : 0);
        const int lpr = gu.natoms * 64 * esz / 128;  // 128-byte lines per row segment
        const uint8_t* base = wb + r0 * rb + (size_t)gu.katom0 * 64 * esz;
#pragma unroll 4
        for (int i = lane_id(); i < nr * lpr; i += 32) {
          const int r = i / lpr, cidx = i - r * lpr;
          asm volatile("prefetch.global.L2 [%0];" ::"l"(base + (size_t)r * rb + cidx * 128));
        }
      }
    }
  };
  if (ahead > 0)
    for (int g = 0; g < ahead && g < total_layers; ++g) prefetch_layer(g);
#pragma unroll 1
  for (int step = 0; ok && step < nsteps; ++step)
#pragma unroll 1
    for (int l = 0; ok && l < L; ++l) {
      if (ahead > 0) prefetch_layer(step * L + l + ahead);
      __syncwarp();
#pragma unroll 1
      for (int m = 0; ok && m < Model::kMats; ++m) {
        const int rows = Model::rows(m);
        for (int u = 0; ok && u < gcnt[m]; ++u) {
          const GemmUnit gu = gul[m][u];
          // half-row units: 64-row boxes of 2 x wg atoms (the same slot bytes)
          const int aps = gu.half ? 2 * wg : wg;
          const int map = gu.half ? Model::wmap_half(m) : Model::wmap(m);
          const int row0 = l * rows + gu.mtile * 128 + (gu.half == 2 ? 64 : 0);
#pragma unroll 1
          for (int j = 0; j < gu.natoms; j += aps, ++it) {
              const int slot = it % R, round = it / R;
              if (round > 0 && !mbar_wait(&bars->wempty[slot], (round - 1) & 1, err, KERR_PRODUCER)) {
                ok = false;
                break;
              }
              if (leader()) {
#ifdef FA_TRACE
                if (trace && u == 0 && j == 0 && step == tstep && l == tlayer) {
                  const int stg = Model::trace_stage(m);
                  trace[((size_t)stg * gridDim.x + blockIdx.x) * kTrStride + kTrProdIssue] = clock64();
                }
#endif
                mbar_expect_tx(&bars->wfull[slot], slot_bytes);
                tma_load_3d(ring + (size_t)slot * slot_bytes, maps + map, &bars->wfull[slot], 0, row0,
                            F8 ? (gu.katom0 + j) >> 1 : gu.katom0 + j, pol);
              }
              __syncwarp();
            }
        }
      }
    }
  // Drain: never leave a TMA write into shared memory in flight at exit.
  const uint32_t first = it > (uint32_t)R ? it - R : 0;
  for (uint32_t k = first; k < it; ++k) mbar_wait(&bars->wfull[k % R], (k / R) & 1, err, KERR_PRODUCER);
}

// ------------------------------------------------------------------ FP8 -> bf16 conversion (epilogue warps)
// Two E4M3 codes -> two bf16 (the bytes that `sel` picks from w: 0x1404 = bytes 0, 1; 0x3424 =
// bytes 2, 3; the lower byte lands in the lower half). Exact, on the integer and bf16x2 pipes:
// prmt places byte b at bits 8..15 of its half; sign | magnitude >> 4 is the bf16 whose value
// is the E4M3 value x 2^-120 (E4M3 subnormals become bf16 subnormals, the same 2^-120 apart);
// the bf16x2 multiply by 2^120 (0x7B80) rescales both exactly.
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2(uint32_t w, uint32_t sel) {
  uint32_t t, out;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(t) : "r"(w), "r"(sel));
  const uint32_t bits = ((t >> 4) & 0x07F007F0u) | (t & 0x80008000u);
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(out) : "r"(bits), "r"(0x7B807B80u));
  return out;
}

// ------------------------------------------------------------------ warp 1 lane 0: GEMM MMAs
// MMA-lane state; lives in shared memory (one instance per CTA, touched by one thread).
struct MmaState {
  uint32_t wit;          // weight-ring slots consumed
  uint32_t bload;        // activation batches loaded (phase of bfull)
  uint32_t bfree;        // activation batches released (phase of bempty)
  uint32_t acc;          // accumulator buffers used
  uint32_t nq, nu;       // attention: Q loads, units
  int last_q;
  uint32_t ns, npv;      // whole-unit attention: S tiles computed, P V products issued
  int k_pre;             // the next attention unit's prefix K is already loading (prefetched)
  uint32_t xu, xc;       // MolmoAct2 whole-unit cross-attention: units, key chunks
  uint32_t qtm;          // token-major GEMMs: activation K-chunks consumed (staging slot phases)
};

// Activation operand of one (unit, token group): atoms [j0, j1) of K x nt token tiles, all
// on ONE barrier so the MMA lane pays a single wait per batch. Item (j, i) sits at
// work + ((j - j0) * nt + i) * tile bytes.
// Register copy of what the GEMM MMA loop needs (see run_producer for why).
struct MmaCtx {
  uint8_t* ring;
  uint8_t* work;
  Bars* bars;
  int* err;
  const CUtensorMap* amap;
  uint32_t tmem;
  int R, batoms, NTILE, TG, tiles, box_atoms, wg;
};

// Activation operand of one (unit, token group): atoms [j0, j1) of K x nt token tiles, all
// on ONE barrier so the MMA lane pays a single wait per batch. Item (j, i) sits at
// work + ((j - j0) * nt + i) * tile bytes.
__device__ __forceinline__ void load_b_batch(const MmaCtx& k, const GemmUnit& gu, int g, int nt, int j0, int j1) {
  if (!leader()) return;
  const uint32_t tile = k.NTILE * 128;
  mbar_expect_tx(&k.bars->bfull, (uint32_t)((j1 - j0) * nt) * tile);
  const uint64_t pol = policy_evict_last();
  const int y0 = g * k.TG * k.NTILE;
  // tile-major: item (j, i) at work + (i * (j1 - j0) + (j - j0)) * tile; one 3D box = box_atoms atoms
#pragma unroll 1
  for (int i = 0; i < nt; ++i)
#pragma unroll 1
    for (int j = j0; j < j1; j += k.box_atoms)
      tma_load_3d(k.work + (size_t)(i * (j1 - j0) + (j - j0)) * tile, k.amap, &k.bars->bfull, 0, y0 + i * k.NTILE,
                  gu.katom0 + j, pol);
}

template <class Model>
__device__ __forceinline__ bool mma_gemm(const typename Model::Params& p, const Ctx& c, MmaState& st_shared, int m) {
  FA_ONE(trace_mark(12));
  MmaState st = st_shared;  // identical copy in every lane; lane 0 writes it back
  MmaCtx k;
  constexpr bool F8 = Model::kF8;  // A from the TMEM slots the epilogue warps fill
  k.ring = c.ring; k.work = c.work; k.bars = c.bars; k.err = p.err; k.amap = &p.maps[Model::act_map(m)];
  k.tmem = c.tmem; k.R = F8 ? kASlotsF8 : c.ring_slots; k.batoms = c.batoms; k.NTILE = p.NTILE; k.TG = p.tg[m];
  k.tiles = p.NPAD / p.NTILE;
  k.box_atoms = p.box_atoms;
  k.wg = p.wg;
  const GemmUnit* const units = c.gu[m];
  const int nunits = c.gcnt[m];
  const uint32_t idesc = idesc_bf16(128, k.NTILE);
  const uint32_t tile = k.NTILE * 128;
  const uint32_t tile16 = tile >> 4;
  const uint32_t slot_bytes = (uint32_t)k.wg * kAtomBytes;
  const uint64_t ring_desc = sdesc_sw128(k.ring), work_desc = sdesc_sw128(k.work);
  Bars* const bars = k.bars;
  uint64_t* const wfull = F8 ? bars->afull : bars->wfull;  // weight slots the MMAs read
  uint64_t* const wempty = F8 ? bars->aempty : bars->wempty;
  #pragma unroll 1
  for (int u = 0; u < nunits; ++u) {
    const GemmUnit gu = units[u];
        {
      const int g = gu.grp;
      const int nt = min(k.TG, k.tiles - g * k.TG);
      // K atoms per activation batch: whole activation boxes (the host sizes the area for one)
      // (and whole weight slots: both granules are powers of two, so their max is a multiple of each)
      const int aps = gu.half ? 2 * k.wg : k.wg;  // weight atoms per ring slot
      const int gran = max(k.box_atoms, aps);
      const int per_batch = max(gran, (k.batoms / nt) / gran * gran);
      int j1 = min((int)gu.natoms, per_batch);
      if (u == 0 && g == 0) FA_ONE(trace_mark(13));
      load_b_batch(k, gu, g, nt, 0, j1);
      if (u == 0 && g == 0) FA_ONE(trace_mark(kTrMmaPre));
      const int a = st.acc & 1;
      if (st.acc >= 2 && !mbar_wait(&bars->acc_empty[a], ((st.acc >> 1) - 1) & 1, k.err, KERR_MMA)) return false;
      tc_fence_after();
      const uint32_t tacc = k.tmem + a * (F8 ? kAccColsF8 : 256);
      #pragma unroll 1
      for (int j0 = 0; j0 < gu.natoms;) {
        if (!mbar_wait(&bars->bfull, st.bload & 1, k.err, KERR_MMA)) return false;
        ++st.bload;
        if (u == 0 && g == 0 && j0 == 0) FA_ONE(trace_mark(kTrMmaB0));
        // A operand of atom jj: a 128-row SW128 tile (16 KB); a half-row unit's 64-row atoms are
        // 8 KB apart, so rows 64..127 of each MMA read the next atom (results ignored)
        const uint32_t astride16 = (gu.half ? kAtomBytes / 2 : kAtomBytes) >> 4;
        int deferred = -1;
#pragma unroll 1
        for (int j = j0; j < j1; j += aps) {  // one ring slot = aps weight atoms
          const int wslot = st.wit % k.R;
          // The last slot before a further activation batch is released only after that batch's
          // loads are issued: otherwise the producer's refill of the slot (the next stage's
          // weights, from HBM) goes out first and the activation batch queues behind it.
          const bool defer = j + aps >= j1 && j1 < gu.natoms;
          if (!mbar_wait(&wfull[wslot], (st.wit / k.R) & 1, k.err, KERR_MMA)) return false;
          if (F8) tc_fence_after();  // the slot's tcgen05.st writes precede these MMAs
          if (u == 0 && g == 0 && j == 0) FA_ONE(trace_mark(kTrMmaW0));
          if (u == 0 && g == 0 && j == 4) FA_ONE(trace_mark(9));
          if (u == 0 && g == 0 && j == 8) FA_ONE(trace_mark(10));
          if (u == 0 && g == 0 && j == 12) FA_ONE(trace_mark(11));
          if (leader()) {
            // Descriptors advance by plain adds from per-slot bases (16-byte units): a per-MMA
            // recomputation leaves the single issuing thread latency-bound, far below the MMA rate.
            const uint64_t da0 = ring_desc + (uint64_t)((wslot * slot_bytes) >> 4);
            const uint32_t ta0 = k.tmem + kAColF8 + wslot * kASlotColsF8;  // FP8: atom = 32 TMEM columns
            const uint64_t db0 = work_desc + (uint64_t)((uint32_t)(j - j0) * tile16);
            const uint32_t bstride16 = (uint32_t)(j1 - j0) * tile16;  // next token tile of the batch
            #pragma unroll 1
            for (int jj = 0; jj < aps; ++jj) {
              const uint64_t da = da0 + (uint64_t)(jj * astride16);
              const uint32_t ta = ta0 + jj * 32;
              const uint64_t dbj = db0 + (uint64_t)(jj * tile16);
              const bool acc0 = (j + jj) != 0;
#pragma unroll
              for (int i = 0; i < 4; ++i) {  // token tiles of the group (<= 4: 256 accumulator columns)
                if (i < nt) {
                  const uint64_t db = dbj + (uint64_t)(i * bstride16);
#pragma unroll
                  for (int s = 0; s < 4; ++s) {
                    if (F8)
                      tc_mma_bf16_ts(tacc + i * k.NTILE, ta + 8 * s, db + 2 * s, idesc, acc0 || s != 0);
                    else
                      tc_mma_bf16(tacc + i * k.NTILE, da + 2 * s, db + 2 * s, idesc, acc0 || s != 0);
                  }
                }
              }
            }
            if (!defer) tc_commit(&wempty[wslot]);
          }
          if (u == 0 && g == 0 && j == 0) FA_ONE(trace_mark(15));
          __syncwarp();
          if (defer) deferred = wslot;
          ++st.wit;
        }
        j0 = j1;
        if (j0 < gu.natoms) {  // reuse the activation area: wait for this batch's MMAs first
          FA_ONE(tc_commit(&bars->bempty));
          if (!mbar_wait(&bars->bempty, st.bfree & 1, k.err, KERR_MMA)) return false;
          ++st.bfree;
          if (u == 0 && g == 0) FA_ONE(trace_mark(14));
          j1 = min((int)gu.natoms, j0 + per_batch);
          load_b_batch(k, gu, g, nt, j0, j1);
          // the deferred slot's MMAs are complete (bempty above covers them)
          if (deferred >= 0) FA_ONE(mbar_arrive(&wempty[deferred]));
        }
      }
      FA_ONE(tc_commit(&bars->acc_full[a]));
      ++st.acc;
    }
  }
  // The next stage overwrites the activation area: its TMA loads must follow these MMAs.
  FA_ONE(tc_commit(&bars->bempty));
  if (!mbar_wait(&bars->bempty, st.bfree & 1, k.err, KERR_MMA)) return false;
  ++st.bfree;
  FA_ONE(trace_mark(kTrMmaDone));
  if (leader()) st_shared = st;
  __syncwarp();
  return true;
}

// ------------------------------------------------------------------ token-major GEMMs (one 64-token tile)
// While the bound batch is a single tile of at most 64 tokens, the GEMMs run "token-major": the
// activation tile is the A operand (M = 64: the tokens), the weights the B operand straight from
// the ring (N = 64 or 128 weight rows), both read from shared memory by the MMA (K-major, 128-byte
// swizzle). Per M64 N64 K16 instruction that is 2 KB of activation and 2 KB of weights.
//
// Activation K-chunks of kTmChunkAtoms atoms (256 K, 64 rows x 128 bytes per atom) are loaded by
// TMA into up to four staging slots and read there by the MMAs; an MMA commit releases a slot. A
// unit's first chunks go out at once, one per slot; a later chunk reuses the slot of the chunk
// before last once that chunk's MMAs have completed.
// (Copying each chunk into tensor memory first and reading A from there was measured slower: the
// epilogue warps' tcgen05.st traffic and the MMAs' tensor-memory reads slowed each other to ~96
// cycles per M128 N64 K16 MMA and ~2,200 cycles per 32 KB chunk.)
// M = 64 accumulator layout: row r in TMEM lane 32 (r >> 4) + (r & 15), one column per weight row.
// TMEM: one accumulator at columns [0, 128) (N <= 128).
// (kTmChunkAtoms, kTmChunkBytes: fa_engine_types.cuh)

// MMAs of NA consecutive weight atoms of one ring slot against the matching activation atoms of a
// staging slot, fully unrolled with compile-time descriptor offsets and issued by one elected lane
// of the converged MMA warp. `first`: the unit's first slot (its first MMA overwrites the
// accumulator).
template <int NA, uint32_t WST16>
__device__ __forceinline__ void tm_issue(uint32_t tacc, uint64_t da, uint64_t db, uint32_t idesc, bool first) {
  constexpr uint32_t kAst16 = 64 * 128 / 16;  // activation atom stride, 16-byte units
#pragma unroll
  for (int jj = 0; jj < NA; ++jj)
#pragma unroll
    for (int s = 0; s < 4; ++s)
      tc_mma_bf16_elect(tacc, da + (uint64_t)(jj * kAst16 + 2 * s), db + (uint64_t)(jj * WST16 + 2 * s), idesc,
                        (jj | s) != 0 || !first);
}

// The MMA warp of a token-major GEMM stage (all 32 lanes: waits on every lane, TMA issue on lane 0,
// MMAs and commits on the elected lane). Ring slots hold 32 KB boxes (wg = 2): one K-chunk of a
// 64-row unit is one slot of 4 atoms, one K-chunk of a 128-row unit two slots of 2 atoms.
template <class Model>
__device__ __forceinline__ bool mma_gemm_tm(const typename Model::Params& p, const Ctx& c, MmaState& st_shared, int m) {
  FA_ONE(trace_mark(12));  // entry
  MmaState st = st_shared;
  uint8_t* const ring = c.ring;
  Bars* const bars = c.bars;
  int* const err = p.err;
  const uint32_t tmem = c.tmem;
  const int R = c.ring_slots;
  constexpr uint32_t kSlotBytes = 2 * kAtomBytes;
  constexpr uint32_t kHalfAtom16 = kAtomBytes / 2 / 16, kFullAtom16 = kAtomBytes / 16;  // weight atom strides
  uint8_t* const work = c.work;
  const CUtensorMap* const amap = &p.maps[Model::act_map(m)];
  const uint64_t pol = policy_evict_last();
  const uint32_t nst = (uint32_t)c.tm_slots;
  const GemmUnit* const units = c.gu[m];
  const int nunits = c.gcnt[m];
  const uint64_t ring_desc = sdesc_sw128(ring), work_desc = sdesc_sw128(work);
  uint32_t wslot = st.wit % R, wphase = (st.wit / R) & 1;
  auto take_slot = [&](uint64_t& db) -> bool {
    if (!mbar_wait(&bars->wfull[wslot], wphase, err, KERR_MMA)) return false;
    db = ring_desc + (uint64_t)((wslot * kSlotBytes) >> 4);
    return true;
  };
  auto release_slot = [&]() {
    tc_commit_elect(&bars->wempty[wslot]);
    ++st.wit;
    if (++wslot == (uint32_t)R) { wslot = 0; wphase ^= 1; }
  };
  // activation chunk q (count over the launch) into staging slot q % nst, once the MMAs of the
  // chunk that used the slot before have completed
  auto load_chunk = [&](uint32_t q, int katom) -> bool {
    const uint32_t sl = q % nst;
    if (q >= nst && !mbar_wait(&bars->sempty[sl], ((q / nst) - 1) & 1, err, KERR_MMA)) return false;
    FA_ONE(mbar_expect_tx(&bars->sfull[sl], kTmChunkBytes));
    FA_ONE(tma_load_3d(work + sl * kTmChunkBytes, amap, &bars->sfull[sl], 0, 0, katom, pol));
    return true;
  };
#pragma unroll 1
  for (int u = 0; u < nunits; ++u) {
    const GemmUnit gu = units[u];
    const int nch = gu.natoms / kTmChunkAtoms;
    const uint32_t q0 = st.qtm;
#pragma unroll 1
    for (int ch = 0; ch < (int)nst && ch < nch; ++ch)
      if (!load_chunk(q0 + ch, gu.katom0 + ch * kTmChunkAtoms)) return false;
    // one accumulator: the previous unit's must have been drained
    if (st.acc >= 1 && !mbar_wait(&bars->acc_empty[0], (st.acc - 1) & 1, err, KERR_MMA)) return false;
#pragma unroll 1
    for (int ch = 0; ch < nch; ++ch) {
      const uint32_t q = q0 + ch, sl = q % nst;
      if (!mbar_wait(&bars->sfull[sl], (q / nst) & 1, err, KERR_MMA)) return false;
      tc_fence_after();
      if (u == 0 && ch < 4) FA_ONE(trace_mark(1 + ch));  // chunk ch landed
      const uint64_t da = work_desc + (uint64_t)((sl * kTmChunkBytes) >> 4);
      uint64_t db;
      if (gu.half) {  // N = 64: 64-row weight atoms of 8 KB, one ring slot per chunk
        if (!take_slot(db)) return false;
        if (u == 0 && ch < 4) FA_ONE(trace_mark(8 + ch));  // its weight slot ready
        tm_issue<4, kHalfAtom16>(tmem, da, db, idesc_bf16(64, 64), ch == 0);
        release_slot();
      } else {  // N = 128: 128-row weight atoms of 16 KB, two ring slots per chunk
        if (!take_slot(db)) return false;
        tm_issue<2, kFullAtom16>(tmem, da, db, idesc_bf16(64, 128), ch == 0);
        release_slot();
        if (!take_slot(db)) return false;
        tm_issue<2, kFullAtom16>(tmem, da + (uint64_t)(2 * 64 * 128 / 16), db, idesc_bf16(64, 128), false);
        release_slot();
      }
      tc_commit_elect(&bars->sempty[sl]);
      if (u == 0 && ch < 3) FA_ONE(trace_mark(13 + ch));  // its MMAs issued
      // the chunk before this one is done with its slot soon: refill it while these MMAs run
      if (ch >= 1 && ch - 1 + (int)nst < nch && !load_chunk(q - 1 + nst, gu.katom0 + (ch - 1 + nst) * kTmChunkAtoms))
        return false;
    }
    st.qtm = q0 + nch;
    tc_commit_elect(&bars->acc_full[0]);
    ++st.acc;
  }
  if (leader()) st_shared = st;
  __syncwarp();
  return true;
}

// Epilogue warps of a token-major GEMM stage: per unit, drain the accumulator through
// Model::epi_tm (thread = token: lanes 0..15 of each warp hold the 16 rows of its lane quadrant;
// 32 weight-row columns at a time).
template <class Model>
__device__ __forceinline__ uint32_t epi_gemm_tm(const typename Model::Params& p, const Ctx& c, uint32_t ecnt, int m,
                                                int l) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3;
  const bool active = lane < 16;
  const int tok = qd * 16 + lane;
  int* const err = p.err;
  Bars* const bars = c.bars;
  const uint32_t tl = c.tmem + ((uint32_t)(qd * 32) << 16);
  const GemmUnit* const units = c.gu[m];
  const int nunits = c.gcnt[m];
  typename Model::Epi e;
  Model::epi_load(e, p, c, l);
#pragma unroll 1
  for (int u = 0; u < nunits; ++u) {
    const GemmUnit gu = units[u];
    if (!mbar_wait(&bars->acc_full[0], ecnt & 1, err, KERR_EPI)) return ecnt;
    tc_fence_after();
    const int ncols = gu.half ? 64 : 128;
#pragma unroll 1
    for (int c0 = 0; c0 < ncols; c0 += 32) {
      float v[32];
      tmem_ld16(tl + c0, v);
      tmem_ld16(tl + c0 + 16, v + 16);
      tc_wait_ld();
      if (active) Model::epi_tm(e, gu, m, tok, c0, v);
    }
    tc_fence_before();
    mbar_arrive(&bars->acc_empty[0]);
    ++ecnt;
  }
  return ecnt;
}

// GEMM epilogue driver (warps 2-5): waits for each accumulator, walks it in 16-token chunks
// through Model::epi_tile and, for staged outputs, copies each 64-token sub-tile out with
// Model::epi_copy_out. Each model hook has ONE call site: instruction-cache space is a
// first-order cost in a persistent kernel whose per-layer code cycles through every stage.
// (A K-split of the RoPE / GeGLU matrices with an in-stage reduction through L2 was measured
// slower than full-K tiles at bs=1: its extra dependent L2 round trips outweigh the shorter MMA
// chains.)
// FP8 streaming: the epilogue warps expand one unit's E4M3 slots into the TMEM A slots, in the
// producer's order. Thread = TMEM lane = row r of the slot's boxes (64-row units: warps of lane
// quadrants 0, 1 only); it reads its row's 16-byte chunks (chunk c of line r at r * 128 +
// ((c ^ (r & 7)) << 4): the 128-byte swizzle), converts 16 codes per chunk and stores a bf16 atom
// (64 K = 32 columns) per tcgen05.st. Every thread, active or not, waits and arrives in order, so
// the barrier phases never run ahead: wfull (slot landed) -> aempty (MMAs done with the A slot)
// -> convert -> wempty (E4M3 slot free) -> afull (A slot written; one arrival per thread).
struct ConvState {
  uint32_t cit;  // E4M3 slots converted so far (the producer's slot sequence)
  int ahead;     // slots of the coming GEMM stage converted ahead, during the barrier before it
};
// Converts slots [s0, s1) of unit gu.
__device__ __forceinline__ bool convert_range(const Ctx& c, int* err, int wg, const GemmUnit& gu, int s0, int s1,
                                              uint32_t& cit) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3;
  const int R = c.ring_slots;
  Bars* const bars = c.bars;
  const int aps = gu.half ? 2 * wg : wg;
  const int nbox = gu.half ? wg : wg / 2;                    // E4M3 boxes per slot (128 K each)
  const uint32_t abytes = gu.half ? 64 * 128 : 128 * 128;    // one box of rows x 128 bytes
  const bool active = gu.half == 0 || qd < 2;
  const int r = qd * 32 + lane;
  const uint32_t fbytes = (uint32_t)wg * kAtomBytes / 2;
  const uint32_t tq = c.tmem + ((uint32_t)(qd * 32) << 16) + kAColF8;
  (void)aps;
#pragma unroll 1
  for (int sl = s0; sl < s1; ++sl, ++cit) {
    const int fslot = cit % R, aslot = cit % kASlotsF8;
    if (!mbar_wait(&bars->wfull[fslot], (cit / R) & 1, err, KERR_EPI)) return false;
    if (cit >= (uint32_t)kASlotsF8 && !mbar_wait(&bars->aempty[aslot], ((cit / kASlotsF8) - 1) & 1, err, KERR_EPI))
      return false;
    tc_fence_after();
    if (active) {
      const uint8_t* src = c.ring + (size_t)fslot * fbytes + r * 128;
#pragma unroll 1
      for (int a = 0; a < 2 * nbox; ++a) {  // bf16 atom a = box a / 2, chunks 4 (a & 1) .. + 3
        uint32_t w[32];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int ch = 4 * (a & 1) + cc;
          const uint4 raw = *reinterpret_cast<const uint4*>(src + (a >> 1) * abytes + ((ch ^ (r & 7)) << 4));
          w[cc * 8 + 0] = e4m3x2_to_bf16x2(raw.x, 0x1404); w[cc * 8 + 1] = e4m3x2_to_bf16x2(raw.x, 0x3424);
          w[cc * 8 + 2] = e4m3x2_to_bf16x2(raw.y, 0x1404); w[cc * 8 + 3] = e4m3x2_to_bf16x2(raw.y, 0x3424);
          w[cc * 8 + 4] = e4m3x2_to_bf16x2(raw.z, 0x1404); w[cc * 8 + 5] = e4m3x2_to_bf16x2(raw.z, 0x3424);
          w[cc * 8 + 6] = e4m3x2_to_bf16x2(raw.w, 0x1404); w[cc * 8 + 7] = e4m3x2_to_bf16x2(raw.w, 0x3424);
        }
        tmem_st32(tq + aslot * kASlotColsF8 + a * 32, w);
      }
    }
    mbar_arrive(&bars->wempty[fslot]);
    if (active) tc_wait_st();
    tc_fence_before();
    mbar_arrive(&bars->afull[aslot]);
  }
  return true;
}

// Converts the first slots of matrix m's units (the next GEMM stage) into the free A slots,
// during the grid barrier before that stage. Every MMA of the stages before has completed by
// then (their accumulators were drained), so the aempty waits do not block.
__device__ __forceinline__ bool convert_ahead(const Ctx& c, int* err, int wg, int m, ConvState& cs) {
  int done = cs.ahead;  // slots of this matrix already converted, from its first unit on
#pragma unroll 1
  for (int u = 0; u < c.gcnt[m] && cs.ahead < kASlotsF8; ++u) {
    const GemmUnit gu = c.gu[m][u];
    const int aps = gu.half ? 2 * wg : wg, ns = (gu.natoms + aps - 1) / aps;
    if (done >= ns) {
      done -= ns;
      continue;
    }
    const int s1 = min(ns, done + (kASlotsF8 - cs.ahead));
    if (!convert_range(c, err, wg, gu, done, s1, cs.cit)) return false;
    cs.ahead += s1 - done;
    done = 0;
  }
  return true;
}

template <class Model>
__device__ __forceinline__ uint32_t epi_gemm(const typename Model::Params& p, const Ctx& c, uint32_t ecnt, int m, int l,
                                             ConvState& cs) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3;
  const int NTILE = p.NTILE, TG = p.tg[m], tiles = p.NPAD / p.NTILE;
  int* const err = p.err;
  Bars* const bars = c.bars;
  const uint32_t taddr = c.tmem + ((uint32_t)(qd * 32) << 16);
  const GemmUnit* const units = c.gu[m];
  const int nunits = c.gcnt[m];
  typename Model::Epi e;
  Model::epi_load(e, p, c, l);
  for (int u = 0; u < nunits; ++u) {
    const GemmUnit gu = units[u];
    const bool staged = Model::staged(m, gu);
    // half-row units: the 64 valid rows sit in TMEM lanes 0..63 (quadrants 0, 1); they are the
    // tile's rows 64 (half - 1) + 0..63, i.e. quadrants qd + 2 (half - 1) of a full tile
    const bool active = gu.half == 0 || qd < 2;
    const int qd_e = gu.half == 2 ? qd + 2 : qd;
    const int row_e = qd_e * 32 + lane;
    // FP8 streaming: the weight row's scale (the MMAs ran on the E4M3 codes)
    // (active rows only: an idle quadrant's row_e can lie past the matrix)
    const float wsc = (Model::kF8 && active) ? Model::row_scale(p, m, l, gu.mtile, row_e) : 1.0f;
    if constexpr (Model::kF8) {  // this unit's slots not already converted ahead
      const int aps = gu.half ? 2 * p.wg : p.wg, ns = (gu.natoms + aps - 1) / aps;
      const int skip = min(cs.ahead, ns);
      cs.ahead -= skip;
      if (!convert_range(c, err, p.wg, gu, skip, ns, cs.cit)) return ecnt;
    }
    {
      const int g = gu.grp;
      const int nchunks = min(TG, tiles - g * TG) * NTILE / 16;
      const int a = ecnt & 1;
      if (!mbar_wait(&bars->acc_full[a], (ecnt >> 1) & 1, err, KERR_EPI)) return ecnt;
      tc_fence_after();
      if (u == 0 && threadIdx.x == 64) trace_mark(kTrEpiAcc0);
      const int tok0 = g * TG * NTILE;
      for (int sub = 0; sub < (nchunks + 3) >> 2; ++sub) {  // 64-token sub-tiles
        const int c0 = sub * 4, c1 = min(nchunks, sub * 4 + 4);
        const int nb0 = tok0 + sub * 64;
#pragma unroll 1
        for (int q = c0; q < c1 && active; ++q) {
          float v[16];
          tmem_ld16(taddr + a * (Model::kF8 ? kAccColsF8 : 256) + q * 16, v);
          tc_wait_ld();
          if (Model::kF8) {
#pragma unroll
            for (int k = 0; k < 16; ++k) v[k] *= wsc;
          }
          Model::epi_tile(e, gu, m, qd_e, lane, row_e, tok0 + q * 16, nb0, v);
        }
        if (staged) {
          sync_epi();
          Model::epi_copy_out(e, gu, m, nb0, 0, (c1 - c0) * 16);
          sync_epi();
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->acc_empty[a]);
      ++ecnt;
    }
  }
  return ecnt;
}

}  // namespace fa
