// pi0.5 flow-matching denoise megakernel for B200 (sm_100a).
//
// One cooperative launch runs all N Euler steps x L expert layers (reference semantics:
// src/pi05/mk6.cu:112-519; Euler schedule benchmarks/pi05/eval_numerics.py:60-68).
//
// CTA = 6 warps, one CTA per SM:
//   warp 0  weight producer: streams this CTA's weight tiles for the WHOLE loop (every step,
//           layer and GEMM stage, in schedule order) through a ring of 16 KB shared-memory
//           slots with TMA. Weights do not depend on activations, so the stream never waits on
//           a grid barrier; only ring space throttles it.
//   warp 1  MMA issuer: one lane issues tcgen05.mma (A = weight tile, B = activation tile,
//           both 128B-swizzled K-major in smem; fp32 accumulators in TMEM) and the TMA loads of
//           activation / attention operands.
//   warps 2-5 epilogue + vector work: TMEM -> registers (tcgen05.ld) -> fused epilogues
//           (RoPE, GeGLU, split-K partials), softmax, adaRMSNorm, merge, final projection.
// Stages of a layer are separated by a bounded grid barrier (a counter in global memory).
#include "fa_pi05.cuh"
#include "fa_ptx.cuh"

namespace fa {
namespace pi05 {

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

// gelu with the tanh approximation (src/pi05/mk6.cu:79-82).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanhf(k0 * (x + 0.044715f * x * x * x)));
}

// Grid barrier among warps 1-5 of every CTA. `gen` counts barriers passed by this launch; the
// counter only grows, so barrier k completes when it reaches (k+1) * gridDim.x. Bounded: on
// timeout (or when another CTA already failed) it raises *err and returns false.
__device__ bool grid_barrier(const Params& p, uint32_t& gen) {
  __shared__ int s_ok;
  sync_main();
  if (threadIdx.x == 32) {
    int ok = 1;
    __threadfence();
    fence_proxy_async_global();
    if (!(blockIdx.x == 0 && (int)gen == p.inject_barrier)) atomicAdd(p.bar, 1u);
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
    __threadfence();
    fence_proxy_async_global();
    s_ok = ok;
  }
  sync_main();
  ++gen;
  return s_ok != 0;
}

// ------------------------------------------------------------------ vector stages (warps 2-5)
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

// adaRMSNorm of one token row already held as 8 values per thread (dims e*4.. and 512+e*4..):
// xn = x * rsqrt(mean(x^2) + 1e-6) * (1 + scale) + shift, stored as bf16 (src/pi05/mk6.cu:139-164).
__device__ __forceinline__ void rms_store(const Params& p, int n, const float v[8], const float* mod, float* red) {
  const int e = threadIdx.x - 64;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  ss = epi_sum(ss, red);
  const float r = rsqrtf(ss * (1.0f / D) + 1e-6f);
#pragma unroll
  for (int hlf = 0; hlf < 2; ++hlf) {
    const int d = hlf * 512 + e * 4;
    const float4 sc = *reinterpret_cast<const float4*>(mod + d);
    const float4 sh = *reinterpret_cast<const float4*>(mod + D + d);
    const float* w = v + hlf * 4;
    __nv_bfloat162 a = __floats2bfloat162_rn(w[0] * r * (1.f + sc.x) + sh.x, w[1] * r * (1.f + sc.y) + sh.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(w[2] * r * (1.f + sc.z) + sh.z, w[3] * r * (1.f + sc.w) + sh.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&a);
    pk.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p.xn + (size_t)n * D + d) = pk;
  }
}

// Loads x[n] and folds in `nsplit` fp32 partials scaled by `gate`: x += gate * sum_s part[s]
// (the gated residual of the previous sub-block, summed in a fixed order: deterministic).
__device__ __forceinline__ void load_residual(const Params& p, int n, const float* gate, int nsplit, float v[8]) {
  const int e = threadIdx.x - 64;
#pragma unroll
  for (int hlf = 0; hlf < 2; ++hlf) {
    const int d = hlf * 512 + e * 4;
    float4 x = __ldcg(reinterpret_cast<const float4*>(p.x + (size_t)n * D + d));
    if (nsplit > 0) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s = 0; s < nsplit; ++s) {
        float4 q = __ldcg(reinterpret_cast<const float4*>(p.part + ((size_t)s * p.NPAD + n) * D + d));
        acc.x += q.x; acc.y += q.y; acc.z += q.z; acc.w += q.w;
      }
      const float4 g = *reinterpret_cast<const float4*>(gate + d);
      x.x += g.x * acc.x; x.y += g.y * acc.y; x.z += g.z * acc.z; x.w += g.w * acc.w;
      *reinterpret_cast<float4*>(p.x + (size_t)n * D + d) = x;
    }
    v[hlf * 4 + 0] = x.x; v[hlf * 4 + 1] = x.y; v[hlf * 4 + 2] = x.z; v[hlf * 4 + 3] = x.w;
  }
}

__device__ __forceinline__ const float* mod_ptr(const Params& p, int step, int l, int which) {
  return p.mods + ((size_t)(step * p.L + l) * 2 + which) * MOD;
}

// norm stage: x += gate * sum(partials); xn = adaRMS(x; mod). One token per CTA iteration.
__device__ void stage_norm(const Params& p, const float* gate, int nsplit, const float* mod, float* red) {
  for (int n = blockIdx.x; n < p.NT; n += gridDim.x) {
    float v[8];
    load_residual(p, n, gate, nsplit, v);
    rms_store(p, n, v, mod, red);
  }
}

// x = W_ain x_t + b_ain for token n (x_t row in smem `xt`), then norm1 of layer 0 of `step`
// (src/pi05/mk6.cu:280-289 then :302).
__device__ void embed_norm_token(const Params& p, int n, int step, const float* xt, float* red) {
  const int e = threadIdx.x - 64;
  float v[8];
#pragma unroll
  for (int hlf = 0; hlf < 2; ++hlf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = hlf * 512 + e * 4 + i;
      float acc = p.b_ain[d];
      const float* w = p.w_ain + (size_t)d * p.AD;
      for (int a = 0; a < p.AD; ++a) acc = fmaf(w[a], xt[a], acc);
      v[hlf * 4 + i] = acc;
    }
    const int d = hlf * 512 + e * 4;
    *reinterpret_cast<float4*>(p.x + (size_t)n * D + d) =
        make_float4(v[hlf * 4 + 0], v[hlf * 4 + 1], v[hlf * 4 + 2], v[hlf * 4 + 3]);
  }
  rms_store(p, n, v, mod_ptr(p, step, 0, 0), red);
}

__device__ void stage_embed(const Params& p, float* xt_s, float* red) {
  const int e = threadIdx.x - 64;
  for (int n = blockIdx.x; n < p.NT; n += gridDim.x) {
    if (e < p.AD) xt_s[e] = p.x_t[(size_t)n * p.AD + e];
    sync_epi();
    embed_norm_token(p, n, 0, xt_s, red);
    sync_epi();
  }
}

// Final adaRMS (mod_final scale|shift), velocity head v = W_aout xn + b, Euler update
// x_t += dt * v (src/pi05/mk6.cu:503-515), then the next step's embed + norm1.
__device__ void stage_final(const Params& p, int step, float* xf, float* xt_s, float* red) {
  const int e = threadIdx.x - 64, lane = e & 31, w = e >> 5;
  const float* gate = mod_ptr(p, step, p.L - 1, 1) + 2 * D;
  const float* modf = p.mod_final + (size_t)step * MOD;
  for (int n = blockIdx.x; n < p.NT; n += gridDim.x) {
    float v[8];
    load_residual(p, n, gate, p.split_dn, v);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
    ss = epi_sum(ss, red);
    const float r = rsqrtf(ss * (1.0f / D) + 1e-6f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = (i >> 2) * 512 + e * 4 + (i & 3);
      xf[d] = v[i] * r * (1.f + modf[d]) + modf[D + d];
    }
    sync_epi();
    for (int a = w; a < p.AD; a += 4) {
      const float* wr = p.w_aout + (size_t)a * D;
      float acc = 0.f;
      for (int d = lane; d < D; d += 32) acc = fmaf(wr[d], xf[d], acc);
      acc = warp_sum(acc);
      if (lane == 0) {
        const float nv = p.x_t[(size_t)n * p.AD + a] + p.dt * (acc + p.b_aout[a]);
        p.x_t[(size_t)n * p.AD + a] = nv;
        xt_s[a] = nv;
      }
    }
    sync_epi();
    if (step + 1 < p.nsteps) embed_norm_token(p, n, step + 1, xt_s, red);
    sync_epi();
  }
}

// Merge the per-chunk attention partials (flash-decoding combine): for each (token, head),
// out = sum_c w_c O_c / sum_c w_c with w_c = exp(m_c - M) l_c.
__device__ void stage_merge(const Params& p) {
  const int e = threadIdx.x - 64;
  const int total = p.NT * H * (HD / 4);
  for (int idx = blockIdx.x * 128 + e; idx < total; idx += gridDim.x * 128) {
    const int n = idx / (H * (HD / 4));
    const int h = (idx / (HD / 4)) % H;
    const int d = (idx % (HD / 4)) * 4;
    const int b = n / p.T, t = n % p.T, hp = h >> 1, r = (h & 1) * TPAD + t;
    const int npc = p.nchunks[b];
    const size_t base = (size_t)(b * 4 + hp) * (MAX_CH + 1);
    float M = -INFINITY;
    for (int c = 0; c <= npc; ++c) {
      const int cc = c < npc ? c : MAX_CH;
      M = fmaxf(M, __ldcg(p.oml + ((base + cc) * 128 + r) * 2));
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float wsum = 0.f;
    for (int c = 0; c <= npc; ++c) {
      const int cc = c < npc ? c : MAX_CH;
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.oml + ((base + cc) * 128 + r) * 2));
      const float wgt = exp2f(ml.x - M) * ml.y;  // max kept in log2 units
      const float4 o = __ldcg(reinterpret_cast<const float4*>(p.opart + ((base + cc) * 128 + r) * HD + d));
      acc.x += wgt * o.x; acc.y += wgt * o.y; acc.z += wgt * o.z; acc.w += wgt * o.w;
      wsum += wgt;
    }
    const float inv = 1.f / wsum;
    __nv_bfloat162 a = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
    __nv_bfloat162 bb = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&a);
    pk.y = *reinterpret_cast<uint32_t*>(&bb);
    *reinterpret_cast<uint2*>(p.attn + (size_t)n * QD + h * HD + d) = pk;
  }
}

// ------------------------------------------------------------------ CTA context
struct Bars {
  uint64_t wfull[kMaxRing], wempty[kMaxRing];
  uint64_t bfull[kBSlots], bempty[kBSlots];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t q_full, k_full, v_full, kv_free, v_free, s_full, p_full, o_full, o_free, drain;
};
struct Ctx {
  uint8_t* ring;   // ring_slots x 16 KB
  uint8_t* work;   // B slots (GEMM) or Q | K/V | P (attention)
  Bars* bars;
  uint32_t tmem;
  int ring_slots;
  const CtaPlan* plan;
};

__host__ __device__ constexpr int mat_rows(int m) {
  return m == MAT_QKV ? QKV_ROWS : (m == MAT_GU ? 2 * F : D);
}
__device__ __forceinline__ int act_map(int m) {
  return m == MAT_O ? MAP_ATTN : (m == MAT_DN ? MAP_H : MAP_XN);
}
__device__ __forceinline__ int group_tiles(const Params& p, int g) {
  const int tiles = p.NPAD / p.NTILE;
  const int rem = tiles - g * p.TG;
  return rem < p.TG ? rem : p.TG;
}

// ------------------------------------------------------------------ warp 0: weight producer
// Walks (step, layer, GEMM matrix, unit, token group, K atom) — the exact order the MMA lane
// consumes — and keeps the ring full. It never waits on activations.
__device__ void run_producer(const Params& p, Ctx& c) {
  const uint64_t pol = policy_evict_first();
  const int R = c.ring_slots;
  uint32_t it = 0;
  bool ok = true;
  for (int step = 0; ok && step < p.nsteps; ++step)
    for (int l = 0; ok && l < p.L; ++l)
      for (int m = 0; ok && m < 4; ++m) {
        const int rows = mat_rows(m);
        for (int u = 0; ok && u < c.plan->g_cnt[m]; ++u) {
          const GemmUnit gu = p.gunits[c.plan->g_off[m] + u];
          for (int g = 0; ok && g < p.ngroups; ++g)
            for (int j = 0; j < gu.natoms; ++j, ++it) {
              const int slot = it % R, round = it / R;
              if (round > 0 && !mbar_wait(&c.bars->wempty[slot], (round - 1) & 1, p.err, KERR_PRODUCER)) {
                ok = false;
                break;
              }
              mbar_expect_tx(&c.bars->wfull[slot], kAtomBytes);
              tma_load_2d(c.ring + (size_t)slot * kAtomBytes, &p.maps[MAP_W_QKV + m], &c.bars->wfull[slot],
                          (gu.katom0 + j) * 64, l * rows + gu.mtile * 128, pol);
            }
        }
      }
  // Drain: never leave a TMA write into shared memory in flight at exit.
  const uint32_t first = it > (uint32_t)R ? it - R : 0;
  for (uint32_t k = first; k < it; ++k) mbar_wait(&c.bars->wfull[k % R], (k / R) & 1, p.err, KERR_PRODUCER);
}

// ------------------------------------------------------------------ warp 1 lane 0: GEMM MMAs
struct MmaState {
  uint32_t wit = 0;       // weight-ring items consumed
  uint32_t bis = 0, bcs = 0;  // activation items issued / consumed
  uint32_t acc = 0;       // accumulator buffers used
  uint32_t nq = 0, nu = 0;  // attention: Q loads, units
  int last_q = -1;
};

__device__ __forceinline__ void issue_b(const Params& p, Ctx& c, MmaState& st, int mapi, int x, int y) {
  const int slot = st.bis % kBSlots, round = st.bis / kBSlots;
  if (round > 0) mbar_wait(&c.bars->bempty[slot], (round - 1) & 1, p.err, KERR_MMA);
  const uint32_t bytes = p.NTILE * 128;
  mbar_expect_tx(&c.bars->bfull[slot], bytes);
  tma_load_2d(c.work + (size_t)slot * (p.NTILE * 128), &p.maps[mapi], &c.bars->bfull[slot], x, y,
              policy_evict_last());
  ++st.bis;
}

__device__ bool mma_gemm(const Params& p, Ctx& c, MmaState& st, int m) {
  const int R = c.ring_slots;
  const uint32_t idesc = idesc_bf16(128, p.NTILE);
  const int mapi = act_map(m);
  for (int u = 0; u < c.plan->g_cnt[m]; ++u) {
    const GemmUnit gu = p.gunits[c.plan->g_off[m] + u];
    for (int g = 0; g < p.ngroups; ++g) {
      const int nt = group_tiles(p, g);
      const int Q = gu.natoms * nt;
      const uint32_t bbase = st.bcs;
      auto item_xy = [&](int k, int& x, int& y) {
        x = (gu.katom0 + k / nt) * 64;
        y = g * p.TG * p.NTILE + (k % nt) * p.NTILE;
      };
      for (int k = 0; k < Q && k < kBSlots - 1; ++k) {
        int x, y;
        item_xy(k, x, y);
        issue_b(p, c, st, mapi, x, y);
      }
      const int a = st.acc & 1;
      if (st.acc >= 2 && !mbar_wait(&c.bars->acc_empty[a], ((st.acc >> 1) - 1) & 1, p.err, KERR_MMA)) return false;
      tc_fence_after();
      const uint32_t tacc = c.tmem + a * 256;
      for (int j = 0; j < gu.natoms; ++j) {
        const int wslot = st.wit % R;
        if (!mbar_wait(&c.bars->wfull[wslot], (st.wit / R) & 1, p.err, KERR_MMA)) return false;
        tc_fence_after();
        const uint64_t da = sdesc_sw128(c.ring + (size_t)wslot * kAtomBytes);
        for (int i = 0; i < nt; ++i) {
          const int k = j * nt + i;
          const uint32_t bq = bbase + k;
          const int bslot = bq % kBSlots;
          if (!mbar_wait(&c.bars->bfull[bslot], (bq / kBSlots) & 1, p.err, KERR_MMA)) return false;
          tc_fence_after();
          const uint64_t db = sdesc_sw128(c.work + (size_t)bslot * (p.NTILE * 128));
#pragma unroll
          for (int s = 0; s < 4; ++s)
            tc_mma_bf16(tacc + i * p.NTILE, da + 2 * s, db + 2 * s, idesc, (j | s) != 0);
          tc_commit(&c.bars->bempty[bslot]);
          if (k + kBSlots - 1 < Q) {
            int x, y;
            item_xy(k + kBSlots - 1, x, y);
            issue_b(p, c, st, mapi, x, y);
          }
        }
        tc_commit(&c.bars->wempty[wslot]);
        ++st.wit;
      }
      st.bcs += Q;
      tc_commit(&c.bars->acc_full[a]);
      ++st.acc;
    }
  }
  return true;
}

// ------------------------------------------------------------------ warps 2-5: GEMM epilogues
// TMEM lane = packed weight row (32 * quadrant + lane), columns = tokens of the tile.
// Packed row orders (host packer) put rotary partners and gate/up partners 16 lanes apart in
// the same warp, so the fused epilogues need one shuffle and no shared memory.
__device__ bool epi_gemm(const Params& p, Ctx& c, uint32_t& ecnt, int m) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3;
  const int row = qd * 32 + lane;
  const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
  for (int u = 0; u < c.plan->g_cnt[m]; ++u) {
    const GemmUnit gu = p.gunits[c.plan->g_off[m] + u];
    for (int g = 0; g < p.ngroups; ++g) {
      const int nt = group_tiles(p, g);
      const int a = ecnt & 1;
      if (!mbar_wait(&c.bars->acc_full[a], (ecnt >> 1) & 1, p.err, KERR_EPI)) return false;
      tc_fence_after();
      for (int i = 0; i < nt; ++i) {
        for (int cc = 0; cc < p.NTILE; cc += 16) {
          float v[16];
          tmem_ld16(c.tmem + lane_addr + a * 256 + i * p.NTILE + cc, v);
          tc_wait_ld();
          const int n0 = g * p.TG * p.NTILE + i * p.NTILE + cc;
          if (m == MAT_QKV) {
            const int mt = gu.mtile;
            if (mt < 18) {  // Q heads (mtile 0..15) or K (16, 17): split-half RoPE epilogue
              const int pb = mt < 16 ? (mt & 1) : mt - 16;
              const int pr = 64 * pb + 16 * qd + (lane & 15);
              const int hi = lane >> 4;
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const float partner = __shfl_xor_sync(0xffffffffu, v[k], 16);
                const int n = n0 + k;
                if (n < p.NT) {
                  const int b = n / p.T, t = n - b * p.T;
                  const float cs = p.rope_cos[(size_t)n * 128 + pr], sn = p.rope_sin[(size_t)n * 128 + pr];
                  const float o = hi ? fmaf(v[k], cs, partner * sn) : fmaf(v[k], cs, -partner * sn);
                  const int dim = pr + 128 * hi;
                  if (mt < 16)
                    p.q[((size_t)(b * H + (mt >> 1)) * TPAD + t) * HD + dim] = __float2bfloat16(o);
                  else
                    p.sk[((size_t)b * TPAD + t) * HD + dim] = __float2bfloat16(o);
                }
              }
            } else {  // V: natural order, stored transposed [dim][token]
              const int dim = (mt - 18) * 128 + row;
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const int n = n0 + k;
                if (n < p.NT) {
                  const int b = n / p.T, t = n - b * p.T;
                  p.svt[((size_t)b * HD + dim) * TPAD + t] = __float2bfloat16(v[k]);
                }
              }
            }
          } else if (m == MAT_GU) {  // GeGLU: lanes 0-15 gate rows, 16-31 up rows of one feature
            const int f = 64 * gu.mtile + 16 * qd + (lane & 15);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const float up = __shfl_xor_sync(0xffffffffu, v[k], 16);
              const int n = n0 + k;
              if (lane < 16 && n < p.NT) p.hbuf[(size_t)n * F + f] = __float2bfloat16(gelu_tanh(v[k]) * up);
            }
          } else {  // O / down: fp32 K-split partial
            float* dst = p.part + ((size_t)gu.split * p.NPAD + n0) * D + gu.mtile * 128 + row;
#pragma unroll
            for (int k = 0; k < 16; ++k) dst[(size_t)k * D] = v[k];
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&c.bars->acc_empty[a]);
      ++ecnt;
    }
  }
  return true;
}

// ------------------------------------------------------------------ attention (split-KV)
// Unit = (observation b, head pair hp, key chunk). 128 query rows = 2 heads x 64 (padded)
// action tokens; the single KV head is shared (MQA). Chunk c < nchunks[b] covers prefix keys
// [128c, 128c+128); the suffix chunk holds this step's 64 (padded) action-token keys.
// S = Q K^T (TMEM cols 0..127) -> softmax rows in registers -> P (bf16, smem) -> O = P V
// (TMEM cols 128..383) -> normalised partial + (max, sum) to global, merged by stage_merge.
constexpr int kQOff = 0, kKVOff = 64 * 1024, kPOff = 128 * 1024;

__device__ bool mma_attn(const Params& p, Ctx& c, MmaState& st, int l) {
  const uint64_t pol_kv = policy_evict_last();
  Bars* br = c.bars;
  for (int u = 0; u < c.plan->a_cnt; ++u) {
    const AttnUnit au = p.aunits[c.plan->a_off + u];
    const int nk = au.is_suffix ? TPAD : KCH;
    const int qkey = au.b * 4 + au.hp;
    if (qkey != st.last_q) {  // previous unit's S MMAs completed (kv_free waited), Q is free
      mbar_expect_tx(&br->q_full, 4 * kAtomBytes);
      for (int a = 0; a < 4; ++a)
        tma_load_2d(c.work + kQOff + a * kAtomBytes, &p.maps[MAP_Q], &br->q_full, a * 64,
                    (au.b * H + 2 * au.hp) * TPAD, pol_kv);
      if (!mbar_wait(&br->q_full, st.nq & 1, p.err, KERR_ATTN)) return false;
      ++st.nq;
      st.last_q = qkey;
    }
    if (st.nu > 0 && !mbar_wait(&br->v_free, (st.nu - 1) & 1, p.err, KERR_ATTN)) return false;
    mbar_expect_tx(&br->k_full, 4 * nk * 128);
    for (int a = 0; a < 4; ++a) {
      if (au.is_suffix)
        tma_load_2d(c.work + kKVOff + a * kAtomBytes, &p.maps[MAP_SK], &br->k_full, a * 64, au.b * TPAD, pol_kv);
      else
        tma_load_2d(c.work + kKVOff + a * kAtomBytes, &p.maps[MAP_K], &br->k_full, a * 64,
                    (au.b * p.L + l) * p.LPAD + au.chunk * KCH, pol_kv);
    }
    if (!mbar_wait(&br->k_full, st.nu & 1, p.err, KERR_ATTN)) return false;
    tc_fence_after();
    const uint32_t id_s = idesc_bf16(128, nk);
    for (int a = 0; a < 4; ++a) {
      const uint64_t dq = sdesc_sw128(c.work + kQOff + a * kAtomBytes);
      const uint64_t dk = sdesc_sw128(c.work + kKVOff + a * kAtomBytes);
#pragma unroll
      for (int s = 0; s < 4; ++s) tc_mma_bf16(c.tmem, dq + 2 * s, dk + 2 * s, id_s, (a | s) != 0);
    }
    tc_commit(&br->s_full);
    tc_commit(&br->kv_free);
    if (!mbar_wait(&br->kv_free, st.nu & 1, p.err, KERR_ATTN)) return false;
    const int nka = nk / 64;  // 64-key atoms
    mbar_expect_tx(&br->v_full, nka * 2 * kAtomBytes);
    for (int kk = 0; kk < nka; ++kk)
      for (int hh = 0; hh < 2; ++hh) {
        uint8_t* dst = c.work + kKVOff + (kk * 2 + hh) * kAtomBytes;
        if (au.is_suffix)
          tma_load_2d(dst, &p.maps[MAP_SVT], &br->v_full, 0, au.b * HD + 128 * hh, pol_kv);
        else
          tma_load_2d(dst, &p.maps[MAP_VT], &br->v_full, au.chunk * KCH + 64 * kk, (au.b * p.L + l) * HD + 128 * hh,
                      pol_kv);
      }
    if (!mbar_wait(&br->v_full, st.nu & 1, p.err, KERR_ATTN)) return false;
    if (!mbar_wait(&br->p_full, st.nu & 1, p.err, KERR_ATTN)) return false;
    if (st.nu > 0 && !mbar_wait(&br->o_free, (st.nu - 1) & 1, p.err, KERR_ATTN)) return false;
    tc_fence_after();
    const uint32_t id_o = idesc_bf16(128, 128);
    for (int kk = 0; kk < nka; ++kk) {
      const uint64_t dp = sdesc_sw128(c.work + kPOff + kk * kAtomBytes);
      for (int hh = 0; hh < 2; ++hh) {
        const uint64_t dv = sdesc_sw128(c.work + kKVOff + (kk * 2 + hh) * kAtomBytes);
#pragma unroll
        for (int s = 0; s < 4; ++s) tc_mma_bf16(c.tmem + 128 + 128 * hh, dp + 2 * s, dv + 2 * s, id_o, (kk | s) != 0);
      }
    }
    tc_commit(&br->o_full);
    tc_commit(&br->v_free);
    ++st.nu;
  }
  return true;
}

__device__ bool epi_attn(const Params& p, Ctx& c, uint32_t& anu) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3;
  const int r = qd * 32 + lane;
  const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
  const float sl2 = 0.0625f * 1.4426950408889634f;  // 1/sqrt(256) in log2 units
  Bars* br = c.bars;
  for (int u = 0; u < c.plan->a_cnt; ++u) {
    const AttnUnit au = p.aunits[c.plan->a_off + u];
    const int nk = au.is_suffix ? TPAD : KCH;
    const int nvalid = au.is_suffix ? p.T : min(KCH, p.valid_len[au.b] - au.chunk * KCH);
    if (!mbar_wait(&br->s_full, anu & 1, p.err, KERR_ATTN)) return false;
    tc_fence_after();
    float mx = -INFINITY;
    for (int cc = 0; cc < nk; cc += 16) {
      float v[16];
      tmem_ld16(c.tmem + lane_addr + cc, v);
      tc_wait_ld();
#pragma unroll
      for (int k = 0; k < 16; ++k)
        if (cc + k < nvalid) mx = fmaxf(mx, v[k] * sl2);
    }
    float sum = 0.f;
    uint8_t* prow = c.work + kPOff + (r >> 3) * 1024 + (r & 7) * 128;
    for (int cc = 0; cc < nk; cc += 16) {
      float v[16];
      tmem_ld16(c.tmem + lane_addr + cc, v);
      tc_wait_ld();
      uint32_t pk[8];
#pragma unroll
      for (int k = 0; k < 16; k += 2) {
        const float p0 = (cc + k < nvalid) ? exp2f(v[k] * sl2 - mx) : 0.f;
        const float p1 = (cc + k + 1 < nvalid) ? exp2f(v[k + 1] * sl2 - mx) : 0.f;
        __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
        sum += __low2float(b2) + __high2float(b2);  // normalise with the probabilities actually used
        pk[k >> 1] = *reinterpret_cast<uint32_t*>(&b2);
      }
      const int atom = cc >> 6, ch = (cc & 63) >> 3;  // two 16-byte chunks of this row
      uint8_t* base = prow + atom * kAtomBytes;
      *reinterpret_cast<uint4*>(base + (((ch) ^ (r & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      *reinterpret_cast<uint4*>(base + (((ch + 1) ^ (r & 7)) << 4)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    }
    fence_proxy_async_shared();
    tc_fence_before();
    mbar_arrive(&br->p_full);
    if (!mbar_wait(&br->o_full, anu & 1, p.err, KERR_ATTN)) return false;
    tc_fence_after();
    const int cidx = au.is_suffix ? MAX_CH : au.chunk;
    const size_t slot = ((size_t)(au.b * 4 + au.hp) * (MAX_CH + 1) + cidx) * 128 + r;
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    float* orow = p.opart + slot * HD;
    for (int cc = 0; cc < HD; cc += 16) {
      float v[16];
      tmem_ld16(c.tmem + lane_addr + 128 + cc, v);
      tc_wait_ld();
#pragma unroll
      for (int k = 0; k < 16; k += 4)
        *reinterpret_cast<float4*>(orow + cc + k) = make_float4(v[k] * inv, v[k + 1] * inv, v[k + 2] * inv, v[k + 3] * inv);
    }
    *reinterpret_cast<float2*>(p.oml + slot * 2) = make_float2(sum > 0.f ? mx : -INFINITY, sum);
    tc_fence_before();
    mbar_arrive(&br->o_free);
    ++anu;
  }
  return true;
}

// ------------------------------------------------------------------ kernel
__global__ void __launch_bounds__(kThreads, 1) pi05_denoise_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars bars;
  __shared__ uint32_t s_tmem;
  __shared__ float s_red[8];
  __shared__ float s_xt[32];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Ctx c;
  c.plan = p.plans + blockIdx.x;
  c.ring_slots = c.plan->ring_slots;
  c.ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  c.work = c.ring + (size_t)c.ring_slots * kAtomBytes;
  c.bars = &bars;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kMaxRing; ++i) { mbar_init(&bars.wfull[i], 1); mbar_init(&bars.wempty[i], 1); }
    for (int i = 0; i < kBSlots; ++i) { mbar_init(&bars.bfull[i], 1); mbar_init(&bars.bempty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&bars.acc_full[i], 1); mbar_init(&bars.acc_empty[i], 128); }
    mbar_init(&bars.q_full, 1); mbar_init(&bars.k_full, 1); mbar_init(&bars.v_full, 1);
    mbar_init(&bars.kv_free, 1); mbar_init(&bars.v_free, 1); mbar_init(&bars.s_full, 1);
    mbar_init(&bars.p_full, 128); mbar_init(&bars.o_full, 1); mbar_init(&bars.o_free, 128);
    mbar_init(&bars.drain, 1);
    fence_mbar_init();
    for (int i = 0; i < NUM_MAPS; ++i) tma_prefetch_desc(&p.maps[i]);
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  c.tmem = s_tmem;

  if (warp == 0) {
    if (lane == 0) run_producer(p, c);
    __syncwarp();
  } else {
    const bool is_mma = (threadIdx.x == 32);
    const bool is_epi = warp >= 2;
    MmaState st;
    uint32_t ecnt = 0, anu = 0, gen = 0;
    uint64_t t_prev = globaltimer();
    const bool timing = p.stage_ns != nullptr && blockIdx.x == 0 && threadIdx.x == 32;
    auto mark = [&](int s) {
      if (timing) {
        const uint64_t t = globaltimer();
        p.stage_ns[s] += t - t_prev;
        t_prev = t;
      }
    };
    // Each stage: role work, then a grid barrier. *err is the single failure signal.
    bool ok = true;
    if (is_epi) stage_embed(p, s_xt, s_red);
    ok = grid_barrier(p, gen);
    mark(ST_NORM1);
    for (int step = 0; ok && step < p.nsteps; ++step) {
      for (int l = 0; ok && l < p.L; ++l) {
        const float* mod_in = mod_ptr(p, step, l, 0);
        const float* mod_post = mod_ptr(p, step, l, 1);
        if (is_mma) mma_gemm(p, c, st, MAT_QKV);
        if (is_epi) epi_gemm(p, c, ecnt, MAT_QKV);
        if (!(ok = grid_barrier(p, gen))) break;
        mark(ST_QKV);
        st.last_q = -1;
        if (is_mma) mma_attn(p, c, st, l);
        if (is_epi) epi_attn(p, c, anu);
        if (!(ok = grid_barrier(p, gen))) break;
        mark(ST_ATTN);
        if (is_epi) stage_merge(p);
        if (!(ok = grid_barrier(p, gen))) break;
        mark(ST_MERGE);
        if (is_mma) mma_gemm(p, c, st, MAT_O);
        if (is_epi) epi_gemm(p, c, ecnt, MAT_O);
        if (!(ok = grid_barrier(p, gen))) break;
        mark(ST_O);
        if (is_epi) stage_norm(p, mod_in + 2 * D, p.split_o, mod_post, s_red);
        if (!(ok = grid_barrier(p, gen))) break;
        mark(ST_NORM2);
        if (is_mma) mma_gemm(p, c, st, MAT_GU);
        if (is_epi) epi_gemm(p, c, ecnt, MAT_GU);
        if (!(ok = grid_barrier(p, gen))) break;
        mark(ST_GU);
        if (is_mma) mma_gemm(p, c, st, MAT_DN);
        if (is_epi) epi_gemm(p, c, ecnt, MAT_DN);
        if (!(ok = grid_barrier(p, gen))) break;
        mark(ST_DN);
        if (l + 1 < p.L) {
          if (is_epi) stage_norm(p, mod_post + 2 * D, p.split_dn, mod_ptr(p, step, l + 1, 0), s_red);
          if (!(ok = grid_barrier(p, gen))) break;
          mark(ST_NORM1);
        } else {
          if (is_epi) stage_final(p, step, reinterpret_cast<float*>(c.work), s_xt, s_red);  // work area idle here
          if (!(ok = grid_barrier(p, gen))) break;
          mark(ST_FINAL);
        }
      }
    }
    if (is_mma) {  // retire every MMA this thread issued before TMEM is released
      tc_commit(&bars.drain);
      mbar_wait(&bars.drain, 0, p.err, KERR_MMA);
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(s_tmem, 512);
  }
}

}  // namespace pi05
}  // namespace fa
