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
#include "fa_engine.cuh"
#include "fa_pi05.cuh"

namespace fa {
namespace pi05 {

// ------------------------------------------------------------------ vector stages (warps 2-5)
// adaRMSNorm of one token row already held as 8 values per thread (dims e*4.. and 512+e*4..):
// xn = x * rsqrt(mean(x^2) + 1e-6) * (1 + scale) + shift, stored as bf16 (src/pi05/mk6.cu:139-164).
__device__ __forceinline__ void rms_store(const Params& p, int n, const float v[8], const float* mod, float* red) {
  const int e = threadIdx.x - 64;
  float4 scs[2], shs[2];
#pragma unroll
  for (int hlf = 0; hlf < 2; ++hlf) {  // issue the modulation reads before the reduction
    scs[hlf] = __ldg(reinterpret_cast<const float4*>(mod + hlf * 512 + e * 4));
    shs[hlf] = __ldg(reinterpret_cast<const float4*>(mod + D + hlf * 512 + e * 4));
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  ss = epi_sum(ss, red);
  const float r = rsqrtf(ss * (1.0f / D) + 1e-6f);
#pragma unroll
  for (int hlf = 0; hlf < 2; ++hlf) {
    const int d = hlf * 512 + e * 4;
    const float4 sc = scs[hlf];
    const float4 sh = shs[hlf];
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
// All loads are issued before any use so the row costs one memory round trip; the partials
// travel by cp.async into the shared scratch `scr` (32 KB) instead of 64 registers.
__device__ __forceinline__ void load_residual(const Params& p, int n, const float* gate, int nsplit, float v[8],
                                              float4* scr) {
  const int e = threadIdx.x - 64;
  float4 x[2], acc[2], g[2];
#pragma unroll
  for (int hlf = 0; hlf < 2; ++hlf) {
    const int d = hlf * 512 + e * 4;
    x[hlf] = __ldcg(reinterpret_cast<const float4*>(p.x + (size_t)n * D + d));
    acc[hlf] = make_float4(0.f, 0.f, 0.f, 0.f);
    g[hlf] = nsplit > 0 ? __ldg(reinterpret_cast<const float4*>(gate + d)) : acc[hlf];
  }
  if (nsplit > 0) {
#pragma unroll
    for (int s = 0; s < 8; ++s)
#pragma unroll
      for (int hlf = 0; hlf < 2; ++hlf)
        if (s < nsplit)  // [split][half][thread]: conflict-free read-back
          cp_async16(scr + (s * 2 + hlf) * 128 + e, p.part + ((size_t)s * p.NPAD + n) * D + hlf * 512 + e * 4);
    cp_async_wait_all();
#pragma unroll
    for (int s = 0; s < 8; ++s)
#pragma unroll
      for (int hlf = 0; hlf < 2; ++hlf)
        if (s < nsplit) {
          const float4 q = scr[(s * 2 + hlf) * 128 + e];
          acc[hlf].x += q.x; acc[hlf].y += q.y; acc[hlf].z += q.z; acc[hlf].w += q.w;
        }
#pragma unroll
    for (int hlf = 0; hlf < 2; ++hlf) {
      x[hlf].x += g[hlf].x * acc[hlf].x; x[hlf].y += g[hlf].y * acc[hlf].y;
      x[hlf].z += g[hlf].z * acc[hlf].z; x[hlf].w += g[hlf].w * acc[hlf].w;
      *reinterpret_cast<float4*>(p.x + (size_t)n * D + hlf * 512 + e * 4) = x[hlf];
    }
  }
#pragma unroll
  for (int hlf = 0; hlf < 2; ++hlf) {
    v[hlf * 4 + 0] = x[hlf].x; v[hlf * 4 + 1] = x[hlf].y; v[hlf * 4 + 2] = x[hlf].z; v[hlf * 4 + 3] = x[hlf].w;
  }
}

__device__ __forceinline__ int tok_b(const Params& p, int n) { return tok_bi(p.invT, n); }

__device__ __forceinline__ const float* mod_ptr(const Params& p, int step, int l, int which) {
  return p.mods + ((size_t)(step * p.L + l) * 2 + which) * MOD;
}

// norm stage: x += gate * sum(partials); xn = adaRMS(x; mod). One token per CTA iteration.
__device__ __forceinline__ void stage_norm(const Params& p, const float* gate, int nsplit, const float* mod, float* red,
                                           float4* scr) {
  for (int n = blockIdx.x; n < p.NT; n += gridDim.x) {
    float v[8];
    load_residual(p, n, gate, nsplit, v, scr);
    if (n == (int)blockIdx.x && threadIdx.x == 64) trace_mark(9);
    rms_store(p, n, v, mod, red);
    if (n == (int)blockIdx.x && threadIdx.x == 64) trace_mark(10);
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

__device__ __noinline__ void stage_embed(const Params& p, float* xt_s, float* red) {
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
__device__ __noinline__ void stage_final(const Params& p, int step, float* xf, float* xt_s, float* red) {
  const int e = threadIdx.x - 64, lane = e & 31, w = e >> 5;
  const float* gate = mod_ptr(p, step, p.L - 1, 1) + 2 * D;
  const float* modf = p.mod_final + (size_t)step * MOD;
  for (int n = blockIdx.x; n < p.NT; n += gridDim.x) {
    float v[8];
    load_residual(p, n, gate, p.split_dn, v, reinterpret_cast<float4*>(xf + 2048));  // scratch after xf
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
// out = sum_c w_c O_c / sum_c w_c with w_c = 2^(m_c - M) l_c (maxima kept in log2 units).
// One warp per (token, head); lane c reads chunk c's (max, sum), lanes own 8 dims each.
__device__ __forceinline__ void stage_merge(const Params& p) {
  // register copies: the asm memory clobbers would force reloads through the references
  const int p_NT = p.NT;
  const int p_T = p.T;
  __nv_bfloat16* const p_attn = p.attn;
  const int* const p_nchunks = p.nchunks;
  float* const p_oml = p.oml;
  __nv_bfloat16* const p_opart = p.opart;
  const float p_invT = p.invT;
  const int e = threadIdx.x - 64, lane = e & 31, wq = e >> 5;
  const int total = p_NT * H;
  constexpr int kFirst = 12;  // chunks per item loaded up front (prefixes up to 1408 keys)
  // One item per warp per pass, its first kFirst partial rows and the (max, sum) pairs in flight
  // together (one round trip). The code is kept small on purpose: every layer runs this stage,
  // and instruction fetches that miss the SM's instruction cache cost an L2 round trip each.
#pragma unroll 1
  for (int item = blockIdx.x * 4 + wq; item < total; item += gridDim.x * 4) {
    const int n = item / H, h = item % H;
    const int b = tok_bi(p_invT, n), t = n - b * p_T, hp = h >> 1;
    const int r = (h & 1) * TPAD + t;
    const int npc = p_nchunks[b], nc = npc + 1;  // prefix chunks + the action-token chunk (stored at MAX_CH)
    const size_t base = (size_t)(b * 4 + hp) * (MAX_CH + 1);
    auto row = [&](int c) {
      const int cc = c < npc ? c : MAX_CH;
      return reinterpret_cast<const uint4*>(p_opart + ((base + cc) * 128 + r) * HD + lane * 8);
    };
    uint4 raw[kFirst];
#pragma unroll
    for (int j = 0; j < kFirst; ++j)
      if (j < nc) raw[j] = __ldcg(row(j));
    float2 ml = make_float2(-INFINITY, 0.f);
    if (lane < nc) {
      const int cc = lane < npc ? lane : MAX_CH;
      ml = __ldcg(reinterpret_cast<const float2*>(p_oml + ((base + cc) * 128 + r) * 2));
    }
    const float M = warp_max(ml.x);
    const float wgt_own = (lane < nc && ml.y > 0.f) ? exp2f(ml.x - M) * ml.y : 0.f;
    const float wsum = warp_sum(wgt_own);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    auto accumulate = [&](const uint4& q, float wgt) {
      const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[k]));
        acc[2 * k] = fmaf(wgt, f.x, acc[2 * k]);
        acc[2 * k + 1] = fmaf(wgt, f.y, acc[2 * k + 1]);
      }
    };
#pragma unroll
    for (int j = 0; j < kFirst; ++j) {
      const float wgt = __shfl_sync(0xffffffffu, wgt_own, j);
      if (j < nc) accumulate(raw[j], wgt);
    }
#pragma unroll 1
    for (int c0 = kFirst; c0 < nc; c0 += 4) {  // longer prefixes: 4 more rows per round trip
      uint4 more[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (c0 + j < nc) more[j] = __ldcg(row(c0 + j));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float wgt = __shfl_sync(0xffffffffu, wgt_own, (c0 + j) & 31);
        if (c0 + j < nc) accumulate(more[j], wgt);
      }
    }
    const float inv = 1.f / wsum;
    uint32_t o4[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(acc[2 * k] * inv, acc[2 * k + 1] * inv);
      o4[k] = *reinterpret_cast<uint32_t*>(&b2);
    }
    *reinterpret_cast<uint4*>(p_attn + (size_t)n * QD + h * HD + lane * 8) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
}

// ------------------------------------------------------------------ warps 2-5: GEMM epilogues
// TMEM lane = packed weight row (32 * quadrant + lane), columns = tokens of the tile.
// Packed row orders (host packer) put rotary partners and gate/up partners 16 lanes apart in
// the same warp, so the fused epilogues need one shuffle and no shared memory.
// Fused epilogue for 16 consecutive tokens (nb..nb+15) of one accumulator row.
// Register copy of the fields the GEMM epilogues touch (see run_producer for why).
struct EpiCtx {
  int NT, T, NPAD;
  float invT;
  const float* rope_cos;
  const float* rope_sin;
  __nv_bfloat16* q;
  __nv_bfloat16* sk;
  __nv_bfloat16* svt;
  __nv_bfloat16* hbuf;
  float* part;
  uint8_t* stage;
};

__device__ __forceinline__ void epi_tile(const EpiCtx& p, const GemmUnit& gu, int m, int qd, int lane, int row, int nb,
                                         int nb0, const float* v) {
  if (m == MAT_QKV) {
    const int mt = gu.mtile;
    if (mt < 18) {  // Q heads (mtile 0..15) or K (16, 17): split-half RoPE epilogue
      const int pb = mt < 16 ? (mt & 1) : mt - 16;
      const int pr = 64 * pb + 16 * qd + (lane & 15);
      const int hi = lane >> 4;
      float cs[16], sn[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {  // batch the table reads before any use
        const int n = min(nb + k, p.NT - 1);
        cs[k] = __ldg(p.rope_cos + (size_t)n * 128 + pr);
        sn[k] = __ldg(p.rope_sin + (size_t)n * 128 + pr);
      }
      float partner[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) partner[k] = __shfl_xor_sync(0xffffffffu, v[k], 16);  // exchanges first
      __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(p.stage) + (nb - nb0) * 128 + (lane & 15) + 16 * qd + 64 * hi;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        // staging row = token within the 64-token sub-tile, 128 dims: (lane & 15) + 16 qd + 64 hi
        const float o = hi ? fmaf(v[k], cs[k], partner[k] * sn[k]) : fmaf(v[k], cs[k], -partner[k] * sn[k]);
        st[k * 128] = __float2bfloat16(o);
      }
    } else {  // V: staged transposed, one 128-byte row of 64 tokens per dim (16-byte chunks
              // swizzled by the row: 4-way bank conflicts instead of 32-way); epi_copy_out writes
              // the rows along the token axis
      uint8_t* srow = p.stage + row * 128;
      const int c = (nb - nb0) >> 3;  // 16 tokens = chunks c, c + 1
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          __nv_bfloat162 b2 = __floats2bfloat162_rn(v[8 * h + 2 * k], v[8 * h + 2 * k + 1]);
          w[k] = *reinterpret_cast<uint32_t*>(&b2);
        }
        *reinterpret_cast<uint4*>(srow + (((c + h) ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  } else if (m == MAT_GU) {  // GeGLU: lanes 0-15 gate rows, 16-31 up rows of one feature
    float up[16], h[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) up[k] = __shfl_xor_sync(0xffffffffu, v[k], 16);  // all exchanges first
#pragma unroll
    for (int k = 0; k < 16; ++k) h[k] = gelu_tanh(v[k]) * up[k];  // 16 independent chains
    if (lane < 16) {  // staging row = token within the sub-tile, 64 features
      __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(p.stage) + (nb - nb0) * 64 + 16 * qd + lane;
#pragma unroll
      for (int k = 0; k < 16; ++k) st[k * 64] = __float2bfloat16(h[k]);
    }
  } else {  // O / down: fp32 K-split partial, each warp store covers 32 consecutive rows
    float* dst = p.part + ((size_t)gu.split * p.NPAD + nb) * D + gu.mtile * 128 + row;
#pragma unroll
    for (int k = 0; k < 16; ++k) dst[(size_t)k * D] = v[k];
  }
}

// Coalesced copy of staged rows (tokens) [r0, r1) of the 64-token sub-tile at nb0 to their
// destination (16-byte stores).
__device__ __forceinline__ void epi_copy_out(const EpiCtx& p, const GemmUnit& gu, int m, int nb0, int r0, int r1) {
  const int e = threadIdx.x - 64;
  // a half-row unit wrote half of the staged row: features / dims of quadrants 2 (half - 1) + {0, 1}
  if (m == MAT_GU) {  // 64 rows (tokens) x 128 B: 8 threads per row
    for (int it = e; it < (r1 - r0) * 8; it += 128) {
      const int t = r0 + (it >> 3), seg = it & 7, n = nb0 + t;
      if (n >= p.NT || (gu.half && (seg >> 2) != gu.half - 1)) continue;
      const uint4 val = *reinterpret_cast<const uint4*>(p.stage + t * 128 + seg * 16);
      *reinterpret_cast<uint4*>(p.hbuf + (size_t)n * F + 64 * gu.mtile + seg * 8) = val;
    }
  } else if (gu.mtile >= 18) {  // V: staged dim rows of 64 tokens -> svt [b][dim][t], two tokens per store
    const int d0 = gu.half ? 64 * (gu.half - 1) : 0, nd = gu.half ? 64 : 128;
    for (int it = e; it < nd * 32; it += 128) {
      const int row = d0 + (it >> 5), tk = r0 + 2 * (it & 31), n = nb0 + tk;
      if (tk >= r1 || n >= p.NT) continue;
      const uint32_t pair = *reinterpret_cast<const uint32_t*>(p.stage + row * 128 + (((tk >> 3) ^ (row & 7)) << 4) + (tk & 7) * 2);
      const int b = tok_bi(p.invT, n), t = n - b * p.T, dim = (gu.mtile - 18) * 128 + row;
      __nv_bfloat16* dst = p.svt + ((size_t)b * HD + dim) * TPAD + t;
      if ((t & 1) == 0 && t + 1 < p.T && n + 1 < p.NT && tk + 1 < r1) {
        *reinterpret_cast<uint32_t*>(dst) = pair;
      } else {  // the pair straddles an observation (odd T) or ends the batch
        dst[0] = __ushort_as_bfloat16((unsigned short)(pair & 0xFFFF));
        if (tk + 1 < r1 && n + 1 < p.NT) {
          const int b1 = tok_bi(p.invT, n + 1), t1 = n + 1 - b1 * p.T;
          p.svt[((size_t)b1 * HD + dim) * TPAD + t1] = __ushort_as_bfloat16((unsigned short)(pair >> 16));
        }
      }
    }
  } else {  // Q / K: 64 rows x 256 B, dims [0, 64) -> 64 pb + ..., dims [64, 128) -> 128 + 64 pb + ...
    const int mt = gu.mtile;
    const int pb = mt < 16 ? (mt & 1) : mt - 16;
    for (int it = e; it < (r1 - r0) * 16; it += 128) {
      const int t = r0 + (it >> 4), seg = it & 15, n = nb0 + t;
      if (n >= p.NT || (gu.half && ((seg & 7) >> 2) != gu.half - 1)) continue;
      const int b = tok_bi(p.invT, n), tt = n - b * p.T;
      const int dim = 64 * pb + (seg & 7) * 8 + (seg >> 3) * 128;
      __nv_bfloat16* dst = mt < 16 ? p.q + ((size_t)(b * H + (mt >> 1)) * TPAD + tt) * HD + dim
                                   : p.sk + ((size_t)b * TPAD + tt) * HD + dim;
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(p.stage + t * 256 + seg * 16);
    }
  }
}

// Token-major epilogue (bound batch = one tile of <= 64 tokens): thread = token n, v = 32
// consecutive columns c0.. of its accumulator row, i.e. 32 consecutive packed weight rows of the
// unit. In the packed QKV and gate/up tiles, row 32 q + i (i < 16) and row 32 q + 16 + i are
// rotary / GeGLU partners, so both halves of a 32-column group sit in this thread's registers.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 b2 = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b2);
}
__device__ __forceinline__ void epi_tm(const EpiCtx& p, const GemmUnit& gu, int m, int n, int c0, const float* v) {
  if (n >= p.NT) return;
  const int q = 2 * (gu.half ? gu.half - 1 : 0) + (c0 >> 5);  // row quadrant of the 128-row packed tile
  if (m == MAT_QKV) {
    const int mt = gu.mtile;
    const int b = tok_bi(p.invT, n), t = n - b * p.T;
    if (mt < 18) {  // Q heads / K: split-half RoPE, pair dims p0 + i and p0 + 128 + i
      const int pb = mt < 16 ? (mt & 1) : mt - 16;
      const int p0 = 64 * pb + 16 * q;
      float cs[16], sn[16];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 c4 = __ldg(reinterpret_cast<const float4*>(p.rope_cos + (size_t)n * 128 + p0) + k);
        const float4 s4 = __ldg(reinterpret_cast<const float4*>(p.rope_sin + (size_t)n * 128 + p0) + k);
        cs[4 * k] = c4.x; cs[4 * k + 1] = c4.y; cs[4 * k + 2] = c4.z; cs[4 * k + 3] = c4.w;
        sn[4 * k] = s4.x; sn[4 * k + 1] = s4.y; sn[4 * k + 2] = s4.z; sn[4 * k + 3] = s4.w;
      }
      uint32_t lo[8], hi[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i0 = 2 * k, i1 = 2 * k + 1;
        lo[k] = pack_bf16x2(fmaf(v[i0], cs[i0], -v[16 + i0] * sn[i0]), fmaf(v[i1], cs[i1], -v[16 + i1] * sn[i1]));
        hi[k] = pack_bf16x2(fmaf(v[16 + i0], cs[i0], v[i0] * sn[i0]), fmaf(v[16 + i1], cs[i1], v[i1] * sn[i1]));
      }
      __nv_bfloat16* dst = mt < 16 ? p.q + ((size_t)(b * H + (mt >> 1)) * TPAD + t) * HD : p.sk + ((size_t)b * TPAD + t) * HD;
      uint4* d0 = reinterpret_cast<uint4*>(dst + p0);
      uint4* d1 = reinterpret_cast<uint4*>(dst + p0 + 128);
      d0[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      d0[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
      d1[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      d1[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
    } else {  // V: natural row order, stored transposed [dim][token]
      const int dim0 = (mt - 18) * 128 + 32 * q;
#pragma unroll
      for (int i = 0; i < 32; ++i) p.svt[((size_t)b * HD + dim0 + i) * TPAD + t] = __float2bfloat16(v[i]);
    }
  } else if (m == MAT_GU) {  // GeGLU: columns i < 16 gate, 16 + i up of feature f0 + i
    const int f0 = 64 * gu.mtile + 16 * q;
    uint32_t hv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      hv[k] = pack_bf16x2(gelu_tanh(v[2 * k]) * v[16 + 2 * k], gelu_tanh(v[2 * k + 1]) * v[17 + 2 * k]);
    uint4* d = reinterpret_cast<uint4*>(p.hbuf + (size_t)n * F + f0);
    d[0] = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    d[1] = make_uint4(hv[4], hv[5], hv[6], hv[7]);
  } else {  // O / down: fp32 K-split partial of rows 32 q .. 32 q + 31 of the tile
    float4* d = reinterpret_cast<float4*>(p.part + ((size_t)gu.split * p.NPAD + n) * D + gu.mtile * 128 + 32 * q);
#pragma unroll
    for (int k = 0; k < 8; ++k) d[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
  }
}

// ------------------------------------------------------------------ model traits for the engine
struct Pi05Model {
  using Params = pi05::Params;
  using Epi = EpiCtx;
  static constexpr int kMats = 4;  // per layer, in consumption order: QKV, O, gate/up, down
  static constexpr bool kF8 = false;
  static constexpr bool kTM = false;  // token-major GEMMs (one tile of <= 64 tokens)
  __device__ static float row_scale(const Params&, int, int, int, int) { return 1.0f; }
  __device__ static int rows(int m) { return m == MAT_QKV ? QKV_ROWS : (m == MAT_GU ? 2 * F : D); }
  __device__ static int wmap(int m) { return MAP_W_QKV + m; }
  __device__ static int wmap_half(int m) { return m == MAT_QKV ? MAP_W_QKV_H : MAP_W_GU_H; }
  __device__ static int act_map(int m) { return m == MAT_O ? MAP_ATTN : (m == MAT_DN ? MAP_H : MAP_XN); }
  __device__ static int trace_stage(int m) {
    return m == MAT_QKV ? ST_QKV : m == MAT_O ? ST_O : m == MAT_GU ? ST_GU : ST_DN;
  }
  __device__ static void epi_load(Epi& e, const Params& p, const Ctx& c, int) {
    e.NT = p.NT; e.T = p.T; e.NPAD = p.NPAD; e.invT = p.invT; e.rope_cos = p.rope_cos; e.rope_sin = p.rope_sin;
    e.q = p.q; e.sk = p.sk; e.svt = p.svt; e.hbuf = p.hbuf; e.part = p.part; e.stage = c.stage;
  }
  __device__ static bool staged(int m, const GemmUnit&) { return m == MAT_GU || m == MAT_QKV; }
  __device__ static void epi_tile(const Epi& e, const GemmUnit& gu, int m, int qd, int lane, int row, int nb, int nb0,
                                  const float* v) {
    pi05::epi_tile(e, gu, m, qd, lane, row, nb, nb0, v);
  }
  __device__ static void epi_copy_out(const Epi& e, const GemmUnit& gu, int m, int nb0, int r0, int r1) {
    pi05::epi_copy_out(e, gu, m, nb0, r0, r1);
  }
  __device__ static void epi_tm(const Epi& e, const GemmUnit& gu, int m, int n, int c0, const float* v) {
    pi05::epi_tm(e, gu, m, n, c0, v);
  }
  // activation operand of matrix m, row-major [NPAD][act_ld(m)] bf16
  __device__ static const __nv_bfloat16* act_src(const Params& p, int m) {
    return m == MAT_O ? p.attn : m == MAT_DN ? p.hbuf : p.xn;
  }
  __device__ static int act_ld(int m) { return m == MAT_O ? QD : m == MAT_DN ? F : D; }
};

// One tile of <= 64 tokens (bs=1 at T <= 64): token-major GEMMs (activations in tensor memory,
// weights as the B operand).
struct Pi05ModelTM : Pi05Model {
  static constexpr bool kTM = true;
};

// FP8 weight streaming: E4M3 tiles in the ring, expanded to bf16 in tensor memory by the epilogue
// warps (the MMAs read A from there), row scales in the epilogue (the reference's W8A16 scheme, src/pi05/mk6.cu:90-94,204-205,219-220).
struct Pi05ModelF8 : Pi05Model {
  static constexpr bool kF8 = true;
  __device__ static float row_scale(const Params& p, int m, int l, int mtile, int row) {
    return __ldg(p.wscale[m] + (size_t)l * rows(m) + mtile * 128 + row);
  }
};

// ------------------------------------------------------------------ attention (split-KV)
// Unit = (observation b, head pair hp, key chunk). 128 query rows = 2 heads x 64 (padded)
// action tokens; the single KV head is shared (MQA). Chunk c < nchunks[b] covers prefix keys
// [128c, 128c+128); the suffix chunk holds this step's 64 (padded) action-token keys.
// S = Q K^T (TMEM cols 0..127) -> softmax rows in registers -> P (bf16, smem) -> O = P V
// (TMEM cols 128..383) -> normalised partial + (max, sum) to global, merged by stage_merge.
constexpr int kQOff = 0, kKVOff = 64 * 1024, kPOff = 128 * 1024;

__device__ __forceinline__ bool mma_attn(const Params& p, const Ctx& c, MmaState& st_shared, int l, bool last) {
  // register copies: the asm memory clobbers would force reloads through the references
  const int c_acnt = c.acnt;
  const AttnUnit* const c_au = c.au;
  Bars* const c_bars = c.bars;
  const uint32_t c_tmem = c.tmem;
  uint8_t* const c_work = c.work;
  const int p_L = p.L;
  const int p_LPAD = p.LPAD;
  int* const p_err = p.err;
  const CUtensorMap* const p_maps = p.maps;
  MmaState st = st_shared;  // identical copy in every lane; lane 0 writes it back
  const uint64_t pol_kv = policy_evict_last();
  Bars* br = c_bars;
  for (int u = 0; u < c_acnt; ++u) {
    const AttnUnit au = c_au[u];
    const int nk = au.is_suffix ? TPAD : KCH;
    const int qkey = au.b * 4 + au.hp;
    // The epilogue stages the previous unit's output in the K/V + P area and then arrives on
    // o_free; nothing may land there (or in TMEM) before that.
    if (st.nu > 0 && !mbar_wait(&br->o_free, (st.nu - 1) & 1, p_err, KERR_ATTN)) return false;
    const bool load_q = qkey != st.last_q;  // Q stays resident across units of one head pair
    if (load_q) {
      FA_ONE(mbar_expect_tx(&br->q_full, 4 * kAtomBytes));
      FA_ONE(tma_load_3d(c_work + kQOff, &p_maps[MAP_Q], &br->q_full, 0, (au.b * H + 2 * au.hp) * TPAD, 0, pol_kv));
    }
    if (st.k_pre) {  // issued at the end of the previous attention stage
      st.k_pre = 0;
    } else {
      FA_ONE(mbar_expect_tx(&br->k_full, 4 * nk * 128));
      if (au.is_suffix)  // atom a of the action-token keys at KV + a * 8 KB
        FA_ONE(tma_load_3d(c_work + kKVOff, &p_maps[MAP_SK], &br->k_full, 0, au.b * TPAD, 0, pol_kv));
      else
        FA_ONE(tma_load_3d(c_work + kKVOff, &p_maps[MAP_K], &br->k_full, 0, (au.b * p_L + l) * p_LPAD + au.chunk * KCH,
                           0, pol_kv));
    }
    if (load_q) {
      if (!mbar_wait(&br->q_full, st.nq & 1, p_err, KERR_ATTN)) return false;
      ++st.nq;
      st.last_q = qkey;
    }
    if (!mbar_wait(&br->k_full, st.nu & 1, p_err, KERR_ATTN)) return false;
    if (u == 0) FA_ONE(trace_mark(kTrMmaW0));  // Q and K in shared memory
    tc_fence_after();
    const uint32_t id_s = idesc_bf16(128, nk);
    for (int a = 0; a < 4; ++a) {
      const uint64_t dq = sdesc_sw128(c_work + kQOff + a * kAtomBytes);
      const uint64_t dk = sdesc_sw128(c_work + kKVOff + a * nk * 128);
#pragma unroll
      for (int s = 0; s < 4; ++s) FA_ONE(tc_mma_bf16(c_tmem, dq + 2 * s, dk + 2 * s, id_s, (a | s) != 0));
    }
    FA_ONE(tc_commit(&br->s_full));
    FA_ONE(tc_commit(&br->kv_free));
    if (!mbar_wait(&br->kv_free, st.nu & 1, p_err, KERR_ATTN)) return false;
    const int nka = nk / 64;  // 64-key atoms
    FA_ONE(mbar_expect_tx(&br->v_full, nka * 2 * kAtomBytes));
    for (int hh = 0; hh < 2; ++hh) {  // V^T atom (dim half hh, key atom kk) at KV + (hh * nka + kk) * 16 KB
      uint8_t* dst = c_work + kKVOff + hh * nka * kAtomBytes;
      if (au.is_suffix)
        FA_ONE(tma_load_3d(dst, &p_maps[MAP_SVT], &br->v_full, 0, au.b * HD + 128 * hh, 0, pol_kv));
      else
        FA_ONE(tma_load_3d(dst, &p_maps[MAP_VT], &br->v_full, 0, (au.b * p_L + l) * HD + 128 * hh, au.chunk * 2, pol_kv));
    }
    if (!mbar_wait(&br->v_full, st.nu & 1, p_err, KERR_ATTN)) return false;
    if (u == 0) FA_ONE(trace_mark(kTrMmaB0));  // V in shared memory
    if (!mbar_wait(&br->p_full, st.nu & 1, p_err, KERR_ATTN)) return false;
    if (u == 0) FA_ONE(trace_mark(10));  // P written by the softmax warps
    tc_fence_after();
    const uint32_t id_o = idesc_bf16(128, 128);
    for (int kk = 0; kk < nka; ++kk) {
      const uint64_t dp = sdesc_sw128(c_work + kPOff + kk * kAtomBytes);
      for (int hh = 0; hh < 2; ++hh) {
        const uint64_t dv = sdesc_sw128(c_work + kKVOff + (hh * nka + kk) * kAtomBytes);
#pragma unroll
        for (int s = 0; s < 4; ++s) FA_ONE(tc_mma_bf16(c_tmem + 128 + 128 * hh, dp + 2 * s, dv + 2 * s, id_o, (kk | s) != 0));
      }
    }
    FA_ONE(tc_commit(&br->o_full));
    ++st.nu;
  }
  // Prefix keys do not change during the loop: once the epilogue has released the K/V area
  // (o_free of the last unit), start loading the first unit's chunk for the next attention stage
  // (layer l + 1, or layer 0 of the next Euler step) so that it is resident when that stage begins.
  if (!last && c_acnt > 0 && !c_au[0].is_suffix) {
    if (!mbar_wait(&br->o_free, (st.nu - 1) & 1, p_err, KERR_ATTN)) return false;
    const AttnUnit au = c_au[0];
    const int ln = (l + 1) % p_L;
    FA_ONE(mbar_expect_tx(&br->k_full, 4 * KCH * 128));
    FA_ONE(tma_load_3d(c_work + kKVOff, &p_maps[MAP_K], &br->k_full, 0, (au.b * p_L + ln) * p_LPAD + au.chunk * KCH, 0,
                       pol_kv));
    st.k_pre = 1;
  }
  FA_ONE(trace_mark(kTrMmaDone));
  if (leader()) st_shared = st;
  __syncwarp();
  return true;
}

// Softmax of one 128-query-row tile over NK keys (one code copy for every NK: each layer runs it,
// and instruction-cache space is a first-order cost), all in one TMEM round trip: thread r owns
// row r (its NK scores in registers), writes the bf16 probabilities as the A operand of O = P V
// (128-byte-swizzled K-major atoms of 64 keys) and returns (max in log2 units, sum).
__device__ __forceinline__ float2 softmax_row(uint32_t taddr, int NK, int nvalid, uint8_t* prow, int r) {
  constexpr float sl2 = 0.0625f * 1.4426950408889634f;  // 1/sqrt(256), log2 units
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
  for (int cc = 0; cc < NK; cc += 32) {  // pass 1: row max, 4 independent chains
    float v[32];
    tmem_ld16(taddr + cc, v);
    tmem_ld16(taddr + cc + 16, v + 16);
    tc_wait_ld();
#pragma unroll
    for (int k = 0; k < 32; ++k)
      if (cc + k < nvalid) m4[k & 3] = fmaxf(m4[k & 3], v[k]);
  }
  const float mraw = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
  const float mx = mraw * sl2;
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
  for (int cc = 0; cc < NK; cc += 32) {  // pass 2: probabilities -> bf16 P atoms
    float v[32];
    tmem_ld16(taddr + cc, v);
    tmem_ld16(taddr + cc + 16, v + 16);
    tc_wait_ld();
    uint32_t pk[16];
#pragma unroll
    for (int k = 0; k < 32; k += 2) {
      const float p0 = cc + k < nvalid ? fast_exp2(fmaf(v[k], sl2, -mx)) : 0.f;
      const float p1 = cc + k + 1 < nvalid ? fast_exp2(fmaf(v[k + 1], sl2, -mx)) : 0.f;
      __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
      s4[(k >> 1) & 3] += __low2float(b2) + __high2float(b2);  // normalise with the stored values
      pk[k >> 1] = *reinterpret_cast<uint32_t*>(&b2);
    }
    uint8_t* base = prow + (cc >> 6) * kAtomBytes;
    const int ch0 = (cc & 63) >> 3;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4*>(base + (((ch0 + q) ^ (r & 7)) << 4)) =
          make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
  }
  return make_float2(mx, (s4[0] + s4[1]) + (s4[2] + s4[3]));
}

constexpr int kOPitch = HD * 2 + 16;  // staged bf16 output row, padded against bank conflicts

__device__ __forceinline__ uint32_t epi_attn(const Params& p, const Ctx& c, uint32_t anu) {
  // register copies: the asm memory clobbers would force reloads through the references
  const int nunits = c.acnt;
  const AttnUnit* const units = c.au;
  Bars* const br = c.bars;
  const uint32_t tmem = c.tmem;
  uint8_t* const work = c.work;
  const int T = p.T;
  int* const err = p.err;
  float* const oml = p.oml;
  __nv_bfloat16* const opart = p.opart;
  const int* const valid_len = p.valid_len;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3;
  const int r = qd * 32 + lane;
  const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
  uint8_t* const stage = work + kKVOff;  // K/V + P area, free once O is in TMEM
  for (int u = 0; u < nunits; ++u) {
    const AttnUnit au = units[u];
    const int nvalid = au.is_suffix ? T : min(KCH, valid_len[au.b] - au.chunk * KCH);
    if (!mbar_wait(&br->s_full, anu & 1, err, KERR_ATTN)) return anu;
    tc_fence_after();
    if (u == 0 && threadIdx.x == 64) trace_mark(kTrEpiAcc0);  // S in TMEM
    uint8_t* prow = work + kPOff + (r >> 3) * 1024 + (r & 7) * 128;
    const float2 ms = softmax_row(tmem + lane_addr, au.is_suffix ? TPAD : KCH, nvalid, prow, r);
    fence_proxy_async_shared();
    tc_fence_before();
    mbar_arrive(&br->p_full);
    if (!mbar_wait(&br->o_full, anu & 1, err, KERR_ATTN)) return anu;
    if (u == 0 && threadIdx.x == 64) trace_mark(11);  // O in TMEM
    tc_fence_after();
    const float inv = ms.y > 0.f ? 1.f / ms.y : 0.f;
    uint8_t* srow = stage + r * kOPitch;
#pragma unroll 1
    for (int cc = 0; cc < HD; cc += 32) {  // normalised O row -> bf16 -> padded staging row
      float v[32];
      tmem_ld16(tmem + lane_addr + 128 + cc, v);
      tmem_ld16(tmem + lane_addr + 128 + cc + 16, v + 16);
      tc_wait_ld();
#pragma unroll
      for (int k = 0; k < 32; k += 8) {
        uint32_t w4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          __nv_bfloat162 b2 = __floats2bfloat162_rn(v[k + 2 * q] * inv, v[k + 2 * q + 1] * inv);
          w4[q] = *reinterpret_cast<uint32_t*>(&b2);
        }
        *reinterpret_cast<uint4*>(srow + (cc + k) * 2) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
    }
    const int cidx = au.is_suffix ? MAX_CH : au.chunk;
    const size_t slot0 = ((size_t)(au.b * 4 + au.hp) * (MAX_CH + 1) + cidx) * 128;
    *reinterpret_cast<float2*>(oml + (slot0 + r) * 2) = make_float2(ms.y > 0.f ? ms.x : -INFINITY, ms.y);
    sync_epi();
    // coalesced copy-out: one 512-byte row per warp instruction
    for (int rr = warp & 3; rr < 128; rr += 4) {
      const uint4 val = *reinterpret_cast<const uint4*>(stage + rr * kOPitch + lane * 16);
      *reinterpret_cast<uint4*>(opart + (slot0 + rr) * HD + lane * 8) = val;
    }
    tc_fence_before();
    mbar_arrive(&br->o_free);
    ++anu;
  }
  return anu;
}

// ------------------------------------------------------------------ attention (whole units, large batches)
// Unit = (observation b, head pair hp) over ALL its key chunks (prefix chunks, then the action-token
// chunk), softmax in two passes: pass 1 computes S = Q K^T chunk by chunk and keeps each query
// row's running maximum; pass 2 recomputes S, forms P = 2^(S - M) with the final maximum M (no
// rescaling of O ever) and accumulates O += P V in tensor memory. The normalised output goes
// straight to `attn`: no per-chunk partials and no merge stage. At large batches this trades one
// extra read of the prefix K and one extra S MMA per chunk for the partial round trip through
// memory (151 MB per layer-step at 64 observations).
__device__ __forceinline__ int whole_chunks(const Params& p, int b) { return p.nchunks[b] + 1; }

__device__ __forceinline__ bool mma_attn_whole(const Params& p, const Ctx& c, MmaState& st_shared, int l) {
  const int c_acnt = c.acnt;
  const AttnUnit* const c_au = c.au;
  Bars* const br = c.bars;
  const uint32_t c_tmem = c.tmem;
  uint8_t* const c_work = c.work;
  const int p_L = p.L, p_LPAD = p.LPAD;
  int* const p_err = p.err;
  const CUtensorMap* const p_maps = p.maps;
  MmaState st = st_shared;
  const uint64_t pol_kv = policy_evict_last();
  for (int u = 0; u < c_acnt; ++u) {
    const AttnUnit au = c_au[u];
    const int nc = whole_chunks(p, au.b);
    // the previous unit's output has been read out of tensor memory
    if (st.nu > 0 && !mbar_wait(&br->o_free, (st.nu - 1) & 1, p_err, KERR_ATTN)) return false;
    FA_ONE(mbar_expect_tx(&br->q_full, 4 * kAtomBytes));
    FA_ONE(tma_load_3d(c_work + kQOff, &p_maps[MAP_Q], &br->q_full, 0, (au.b * H + 2 * au.hp) * TPAD, 0, pol_kv));
    if (!mbar_wait(&br->q_full, st.nq & 1, p_err, KERR_ATTN)) return false;
    ++st.nq;
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
#pragma unroll 1
      for (int ch = 0; ch < nc; ++ch) {
        const bool suffix = ch == nc - 1;
        const int nk = suffix ? TPAD : KCH;
        // K into the K/V area: free once the previous S (pass 1) or P V (pass 2) has run
        FA_ONE(mbar_expect_tx(&br->k_full, 4 * nk * 128));
        if (suffix)
          FA_ONE(tma_load_3d(c_work + kKVOff, &p_maps[MAP_SK], &br->k_full, 0, au.b * TPAD, 0, pol_kv));
        else
          FA_ONE(tma_load_3d(c_work + kKVOff, &p_maps[MAP_K], &br->k_full, 0, (au.b * p_L + l) * p_LPAD + ch * KCH, 0,
                             pol_kv));
        // the S tile in tensor memory has been read by the softmax warps
        if (st.ns > 0 && !mbar_wait(&br->s_free, (st.ns - 1) & 1, p_err, KERR_ATTN)) return false;
        if (!mbar_wait(&br->k_full, st.ns & 1, p_err, KERR_ATTN)) return false;
        tc_fence_after();
        const uint32_t id_s = idesc_bf16(128, nk);
        if (leader()) {
          const uint64_t dq0 = sdesc_sw128(c_work + kQOff), dk0 = sdesc_sw128(c_work + kKVOff);
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            const uint64_t dq = dq0 + (uint64_t)((a * kAtomBytes) >> 4);
            const uint64_t dk = dk0 + (uint64_t)((a * nk * 128) >> 4);
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4) tc_mma_bf16(c_tmem, dq + 2 * s4, dk + 2 * s4, id_s, (a | s4) != 0);
          }
          tc_commit(&br->s_full);
          tc_commit(&br->kv_free);
        }
        __syncwarp();
        if (!mbar_wait(&br->kv_free, st.ns & 1, p_err, KERR_ATTN)) return false;  // S done: K area free
        ++st.ns;
        if (pass == 1) {  // V of this chunk, then O += P V once the softmax warps have written P
          const int nka = nk / 64;
          FA_ONE(mbar_expect_tx(&br->v_full, nka * 2 * kAtomBytes));
          for (int hh = 0; hh < 2; ++hh) {
            uint8_t* dst = c_work + kKVOff + hh * nka * kAtomBytes;
            if (suffix)
              FA_ONE(tma_load_3d(dst, &p_maps[MAP_SVT], &br->v_full, 0, au.b * HD + 128 * hh, 0, pol_kv));
            else
              FA_ONE(tma_load_3d(dst, &p_maps[MAP_VT], &br->v_full, 0, (au.b * p_L + l) * HD + 128 * hh, ch * 2, pol_kv));
          }
          if (!mbar_wait(&br->v_full, st.npv & 1, p_err, KERR_ATTN)) return false;
          if (!mbar_wait(&br->p_full, st.npv & 1, p_err, KERR_ATTN)) return false;
          tc_fence_after();
          const uint32_t id_o = idesc_bf16(128, 128);
          if (leader()) {
            const uint64_t dp0 = sdesc_sw128(c_work + kPOff), dv0 = sdesc_sw128(c_work + kKVOff);
            for (int kk = 0; kk < nka; ++kk)
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const uint64_t dp = dp0 + (uint64_t)((kk * kAtomBytes) >> 4);
                const uint64_t dv = dv0 + (uint64_t)(((hh * nka + kk) * kAtomBytes) >> 4);
#pragma unroll
                for (int s4 = 0; s4 < 4; ++s4)
                  tc_mma_bf16(c_tmem + 128 + 128 * hh, dp + 2 * s4, dv + 2 * s4, id_o, (ch | kk | s4) != 0);
              }
            tc_commit(&br->pv_done);
          }
          __syncwarp();
          if (!mbar_wait(&br->pv_done, st.npv & 1, p_err, KERR_ATTN)) return false;  // K/V area and P free
          ++st.npv;
        }
      }
    }
    FA_ONE(tc_commit(&br->o_full));
    ++st.nu;
  }
  if (leader()) st_shared = st;
  __syncwarp();
  return true;
}

// Row maximum of one S tile over its valid keys (raw scores).
template <int NK>
__device__ __forceinline__ float row_max_s(uint32_t taddr, int nvalid) {
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
  for (int cc = 0; cc < NK; cc += 32) {
    float v[32];
    tmem_ld16(taddr + cc, v);
    tmem_ld16(taddr + cc + 16, v + 16);
    tc_wait_ld();
#pragma unroll
    for (int k = 0; k < 32; ++k)
      if (cc + k < nvalid) m4[k & 3] = fmaxf(m4[k & 3], v[k]);
  }
  return fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
}

// P = 2^(S sl2 - mx) of one S tile as bf16 K-major atoms in shared memory (the A operand of P V);
// returns the row sum of the stored values.
template <int NK>
__device__ __forceinline__ float probs_row(uint32_t taddr, int nvalid, float mx, uint8_t* prow, int r) {
  constexpr float sl2 = 0.0625f * 1.4426950408889634f;
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
  for (int cc = 0; cc < NK; cc += 32) {
    float v[32];
    tmem_ld16(taddr + cc, v);
    tmem_ld16(taddr + cc + 16, v + 16);
    tc_wait_ld();
    uint32_t pk[16];
#pragma unroll
    for (int k = 0; k < 32; k += 2) {
      const float p0 = cc + k < nvalid ? fast_exp2(fmaf(v[k], sl2, -mx)) : 0.f;
      const float p1 = cc + k + 1 < nvalid ? fast_exp2(fmaf(v[k + 1], sl2, -mx)) : 0.f;
      __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
      s4[(k >> 1) & 3] += __low2float(b2) + __high2float(b2);
      pk[k >> 1] = *reinterpret_cast<uint32_t*>(&b2);
    }
    uint8_t* base = prow + (cc >> 6) * kAtomBytes;
    const int ch0 = (cc & 63) >> 3;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4*>(base + (((ch0 + q) ^ (r & 7)) << 4)) =
          make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
  }
  return (s4[0] + s4[1]) + (s4[2] + s4[3]);
}

struct AttnEpiState {
  uint32_t anu, ns, npv;  // units finished, S tiles read, P V products waited for
};

__device__ __forceinline__ void epi_attn_whole(const Params& p, const Ctx& c, AttnEpiState& es) {
  constexpr float sl2 = 0.0625f * 1.4426950408889634f;
  const int nunits = c.acnt;
  const AttnUnit* const units = c.au;
  Bars* const br = c.bars;
  const uint32_t tmem = c.tmem;
  uint8_t* const work = c.work;
  const int T = p.T;
  int* const err = p.err;
  const int* const valid_len = p.valid_len;
  __nv_bfloat16* const attn = p.attn;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3;
  const int r = qd * 32 + lane;
  const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
  uint8_t* const prow = work + kPOff + (r >> 3) * 1024 + (r & 7) * 128;
  for (int u = 0; u < nunits; ++u) {
    const AttnUnit au = units[u];
    const int nc = whole_chunks(p, au.b);
    const int vl = valid_len[au.b];
    float mx = -INFINITY;
    float sum = 0.f;
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
#pragma unroll 1
      for (int ch = 0; ch < nc; ++ch) {
        const bool suffix = ch == nc - 1;
        const int nvalid = suffix ? T : min(KCH, vl - ch * KCH);
        if (!mbar_wait(&br->s_full, es.ns & 1, err, KERR_ATTN)) return;
        tc_fence_after();
        if (pass == 0) {
          const float m = suffix ? row_max_s<TPAD>(tmem + lane_addr, nvalid) : row_max_s<KCH>(tmem + lane_addr, nvalid);
          mx = fmaxf(mx, m);
          tc_fence_before();
          mbar_arrive(&br->s_free);
        } else {
          // P of the previous chunk has been consumed by its P V MMAs
          if (ch > 0 && !mbar_wait(&br->pv_done, (es.npv - 1) & 1, err, KERR_ATTN)) return;
          const float mxs = mx * sl2;
          sum += suffix ? probs_row<TPAD>(tmem + lane_addr, nvalid, mxs, prow, r)
                        : probs_row<KCH>(tmem + lane_addr, nvalid, mxs, prow, r);
          fence_proxy_async_shared();
          tc_fence_before();
          mbar_arrive(&br->s_free);
          mbar_arrive(&br->p_full);
          ++es.npv;
        }
        ++es.ns;
      }
    }
    if (!mbar_wait(&br->o_full, es.anu & 1, err, KERR_ATTN)) return;
    tc_fence_after();
    // row r: head 2 hp + (r >> 6), action token t = r & 63
    const int t = r & 63;
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    __nv_bfloat16* dst = attn + (size_t)(au.b * T + t) * QD + (2 * au.hp + (r >> 6)) * HD;
#pragma unroll 1
    for (int cc = 0; cc < HD; cc += 32) {
      float v[32];
      tmem_ld16(tmem + lane_addr + 128 + cc, v);
      tmem_ld16(tmem + lane_addr + 128 + cc + 16, v + 16);
      tc_wait_ld();
      if (t < T) {
#pragma unroll
        for (int k = 0; k < 32; k += 8) {
          uint32_t w4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(v[k + 2 * q] * inv, v[k + 2 * q + 1] * inv);
            w4[q] = *reinterpret_cast<uint32_t*>(&b2);
          }
          *reinterpret_cast<uint4*>(dst + cc + k) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
    }
    tc_fence_before();
    mbar_arrive(&br->o_free);
    ++es.anu;
  }
}

// ------------------------------------------------------------------ kernel
template <class Model>
__device__ __forceinline__ void denoise_body(const Params& p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars bars;
  __shared__ uint32_t s_tmem;
  __shared__ float s_red[8];
  __shared__ float s_xt[32];
  __shared__ CtaPlan s_plan;
  __shared__ GemmUnit s_gu[kMaxGU];
  __shared__ AttnUnit s_au[kMaxAU];

  __shared__ Ctx s_c;        // per-CTA constants, shared so that no role keeps them on its stack
  __shared__ MmaState s_st;  // MMA-lane state
  const int warp = threadIdx.x >> 5;
  Ctx& c = s_c;
  if (threadIdx.x == 0) {
    s_plan = p.plans[blockIdx.x];
    g_trp = nullptr;
    s_st.wit = s_st.bload = s_st.bfree = s_st.acc = s_st.nq = s_st.nu = 0;
    s_st.last_q = -1;
    s_st.k_pre = 0;
    s_st.ns = s_st.npv = 0;
    s_st.qtm = 0;
  }
  __syncthreads();
  {  // this CTA's work lists, read once from global memory
    int ng = 0;
    for (int m = 0; m < Pi05Model::kMats; ++m) ng += s_plan.g_cnt[m];
    for (int i = threadIdx.x; i < ng; i += blockDim.x) s_gu[i] = p.gunits[s_plan.g_off[0] + i];
    for (int i = threadIdx.x; i < s_plan.a_cnt; i += blockDim.x) s_au[i] = p.aunits[s_plan.a_off + i];
  }
  if (threadIdx.x == 0) {
  for (int m = 0, off = 0; m < Pi05Model::kMats; ++m) {
    c.gu[m] = s_gu + off;
    c.gcnt[m] = s_plan.g_cnt[m];
    off += s_plan.g_cnt[m];
  }
  c.au = s_au;
  c.acnt = s_plan.a_cnt;
  c.batoms = min(kMaxBAtoms, s_plan.b_bytes / (p.NTILE * 128));
  c.ring_slots = s_plan.ring_slots;
  c.tm_slots = min(4, s_plan.b_bytes / (int)kTmChunkBytes);
  c.ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  // ring slots: wg bf16 atoms, or (FP8 streaming) the same K range of E4M3 codes, half the bytes
  c.work = c.ring + (size_t)c.ring_slots * p.wg * (Model::kF8 ? kAtomBytes / 2 : kAtomBytes);
  // epilogue staging: the P area on attention CTAs (idle outside the attention stage), else the
  // 16 KB after the activation area
  c.stage = s_plan.a_cnt > 0 ? c.work + kPOff : c.work + s_plan.b_bytes;
  c.bars = &bars;
  }

  if (threadIdx.x == 0) {
    // E4M3 slots are released by the 128 epilogue threads that convert them, bf16 slots by an
    // MMA commit; TMEM A slots are filled by those threads and released by an MMA commit
    for (int i = 0; i < kMaxRing; ++i) { mbar_init(&bars.wfull[i], 1); mbar_init(&bars.wempty[i], Model::kF8 ? 128 : 1); }
    // A slots: filled by the 128 converting threads (FP8)
    for (int i = 0; i < (int)kTmASlots; ++i) { mbar_init(&bars.afull[i], 128); mbar_init(&bars.aempty[i], 1); }
    for (int i = 0; i < 4; ++i) { mbar_init(&bars.sfull[i], 1); mbar_init(&bars.sempty[i], 1); }
    mbar_init(&bars.bfull, 1);
    mbar_init(&bars.bempty, 1);
    for (int i = 0; i < 2; ++i) { mbar_init(&bars.acc_full[i], 1); mbar_init(&bars.acc_empty[i], 128); }
    mbar_init(&bars.q_full, 1); mbar_init(&bars.k_full, 1); mbar_init(&bars.v_full, 1);
    mbar_init(&bars.kv_free, 1); mbar_init(&bars.v_free, 1); mbar_init(&bars.s_full, 1);
    mbar_init(&bars.p_full, 128); mbar_init(&bars.o_full, 1); mbar_init(&bars.o_free, 128);
    mbar_init(&bars.drain, 1);
    mbar_init(&bars.s_free, 128); mbar_init(&bars.pv_done, 1);
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
  if (threadIdx.x == 0) c.tmem = s_tmem;
  __syncthreads();

  if (warp == 0) {
    run_producer<Model>(p, c);
    __syncwarp();
  } else {
    const bool is_mma = (warp == 1);
    const bool is_epi = warp >= 2;
    MmaState& st = s_st;
    uint32_t ecnt = 0, anu = 0, gen = 0;
    AttnEpiState aes{0, 0, 0};  // whole-unit attention (epilogue warps)
    ConvState cs{0, 0};  // FP8 kernel: E4M3 slots converted (epilogue warps)
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
    auto tr = [&](int stage, int step, int l) -> unsigned long long* {
      if (!p.trace || step != p.trace_step || l != p.trace_layer) return nullptr;
      return p.trace + ((size_t)stage * gridDim.x + blockIdx.x) * kTrStride;
    };
    auto epi_done = [&]() {
      if (threadIdx.x == 64) trace_mark(kTrEpiDone);
    };
    // FP8 kernel: the barrier before a GEMM stage also expands that stage's first weight slots
    // into tensor memory (not before the O projection's stage follows attention, whose TMEM
    // columns overlap the A slots: its slots are expanded during the merge barrier)
    auto ahead = [&](int m) {
      return [&, m]() {
        if constexpr (Model::kF8) {
          if (m >= 0 && p.f8_ahead) convert_ahead(c, p.err, p.wg, m, cs);
        }
      };
    };
    if (is_epi) stage_embed(p, s_xt, s_red);
    ok = grid_barrier(p, gen++, tr(ST_QKV, 0, 0), ahead(MAT_QKV));
    mark(ST_NORM1);
    // One pass of the loop body per stage, each role function reached from ONE call site so
    // that it is inlined: no ABI calls (and no register save / restore through local memory,
    // which misses the small L1 beside 224 KB of shared memory) between stages.
    // Stage order per layer: QKV, attention, merge, O, norm2, gate/up, down, norm1 | final.
    // (selects instead of arrays: a runtime-indexed array would live in local memory)
    auto gemm_of = [](int s) { return s == 0 ? MAT_QKV : s == 3 ? MAT_O : s == 5 ? MAT_GU : s == 6 ? MAT_DN : -1; };
    auto timed = [](int s) {
      return s == 0 ? ST_QKV : s == 1 ? ST_ATTN : s == 2 ? ST_MERGE : s == 3 ? ST_O : s == 4 ? ST_NORM2
           : s == 5 ? ST_GU : s == 6 ? ST_DN : ST_NORM1;
    };
#pragma unroll 1
    for (int step = 0; ok && step < p.nsteps; ++step) {
#pragma unroll 1
      for (int l = 0; ok && l < p.L; ++l) {
        const float* mod_in = mod_ptr(p, step, l, 0);
        const float* mod_post = mod_ptr(p, step, l, 1);
        const bool last_layer = l + 1 == p.L;
#pragma unroll 1
        for (int s = 0; s < 8; ++s) {
          const int m = gemm_of(s);
          if (m >= 0) {
            if constexpr (Model::kTM) {
              if (is_mma) mma_gemm_tm<Model>(p, c, st, m);
              if (is_epi) ecnt = epi_gemm_tm<Model>(p, c, ecnt, m, l);
            } else {
              if (is_mma) mma_gemm<Model>(p, c, st, m);
              if (is_epi) ecnt = epi_gemm<Model>(p, c, ecnt, m, l, cs);
            }
          } else if (s == 1) {
            if (p.attn_whole) {
              if (is_mma) mma_attn_whole(p, c, st, l);
              if (is_epi) epi_attn_whole(p, c, aes);
            } else {
              if (is_mma) {
                if (leader()) st.last_q = -1;
                __syncwarp();
                mma_attn(p, c, st, l, step + 1 == p.nsteps && last_layer);
              }
              if (is_epi) anu = epi_attn(p, c, anu);
            }
          } else if (s == 2) {
            if (is_epi && !p.attn_whole) stage_merge(p);  // whole units wrote attn themselves
          } else if (s == 4 || !last_layer) {  // norm2 | norm1 of the next layer
            if (is_epi) {
              const bool n2 = s == 4;
              // the partials' scratch: the first 32 KB of the work area (idle in a norm stage; on
              // attention CTAs the Q region, clear of the prefetched K)
              stage_norm(p, (n2 ? mod_in : mod_post) + 2 * D, n2 ? p.split_o : p.split_dn,
                         n2 ? mod_post : mod_ptr(p, step, l + 1, 0), s_red, reinterpret_cast<float4*>(c.work));
            }
          } else if (is_epi) {
            stage_final(p, step, reinterpret_cast<float*>(c.work), s_xt, s_red);  // work area idle here
          }
          epi_done();
          // trace / timing ids: the stage that starts after this barrier, the stage that ended
          const int nxt = s < 7 ? timed(s + 1) : ST_QKV;
          const int nstep = s < 7 ? step : (last_layer ? step + 1 : step);
          const int nl = s < 7 ? l : (last_layer ? 0 : l + 1);
          // the GEMM of the next stage, when its expansion may start now
          const int pre = s == 2 ? MAT_O : s == 4 ? MAT_GU : s == 5 ? MAT_DN
                        : (s == 7 && !(last_layer && step + 1 == p.nsteps)) ? MAT_QKV : -1;
          if (!(ok = grid_barrier(p, gen++, tr(nxt == ST_NORM1 && last_layer ? ST_FINAL : nxt, nstep, nl), ahead(pre))))
            break;
          mark(s == 7 && last_layer ? ST_FINAL : timed(s));
        }
      }
    }
    if (is_mma) {  // retire every MMA this warp issued before TMEM is released
      FA_ONE(tc_commit(&bars.drain));
      mbar_wait(&bars.drain, 0, p.err, KERR_MMA);
      if (s_st.k_pre) mbar_wait(&bars.k_full, s_st.nu & 1, p.err, KERR_ATTN);  // no TMA left in flight
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

__global__ void __launch_bounds__(kThreads, 1) pi05_denoise_kernel(const __grid_constant__ Params p) {
  denoise_body<Pi05Model>(p);
}
__global__ void __launch_bounds__(kThreads, 1) pi05_denoise_kernel_f8(const __grid_constant__ Params p) {
  denoise_body<Pi05ModelF8>(p);
}
__global__ void __launch_bounds__(kThreads, 1) pi05_denoise_kernel_tm(const __grid_constant__ Params p) {
  denoise_body<Pi05ModelTM>(p);
}

}  // namespace pi05
}  // namespace fa
