// MolmoAct2 action-expert flow megakernel for B200 (sm_100a).
//
// One cooperative launch runs all N Euler steps x 36 DiT blocks (reference semantics:
// src/molmoact2/mk_ma2.cu:103-576; schedule benchmarks/molmoact2/eval_numerics.py:59-75).
// Per block: adaRMS (self) -> QKV GEMM + bias -> self-attention over the action tokens
// (weightless RMS qk-norm, half-split RoPE over 48 pairs) -> out GEMM + bias, gated residual ->
// adaRMS (cross) -> cross-q GEMM + bias -> cross-attention over the bound context (per-head RMS
// q-norm, split over key chunks, merged) -> out GEMM + bias, gated residual -> adaRMS (mlp) ->
// gate/up GEMM + bias, SiLU gate -> down GEMM + bias, gated residual. Final adaRMS, velocity
// head on the valid action dims, x_t += dt v.
//
// The six GEMMs per block run on the shared tcgen05 engine (fa_engine.cuh): TMA-streamed
// weight tiles, fp32 accumulators in TMEM, fused epilogues. The attention stages are small at
// this horizon (T <= 32) and run on the CUDA cores of the epilogue warps.
#include "fa_engine.cuh"
#include "fa_ma2.cuh"

namespace fa {
namespace ma2 {

constexpr float kEps = 1e-6f;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ int tok_b(const Params& p, int n) { return tok_bi(p.invT, n); }
__device__ __forceinline__ const float* mod_ptr(const Params& p, int step, int l, int norm) {
  return p.mods + ((size_t)(step * p.L + l) * 3 + norm) * MOD;
}

// ------------------------------------------------------------------ norms (warps 2-5)
// A 768-wide row held as 6 values per thread: dims 2e + 256 k + {0, 1}, k = 0..2.
// The partials travel by cp.async into the shared scratch `scr` ([split][3][128] float2, at most
// 36 KB): all of them are in flight at once without holding registers.
__device__ __forceinline__ void row_load_residual(const Params& p, int n, const float* gate, int nsplit,
                                                  float v[6], float2* scr) {
  const int e = threadIdx.x - 64;
  float2 x[3], acc[3], g[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const int d = 2 * e + 256 * k;
    x[k] = __ldcg(reinterpret_cast<const float2*>(p.x + (size_t)n * D + d));
    acc[k] = make_float2(0.f, 0.f);
    g[k] = nsplit > 0 ? __ldg(reinterpret_cast<const float2*>(gate + d)) : acc[k];
  }
  for (int s = 0; s < nsplit; ++s)
#pragma unroll
    for (int k = 0; k < 3; ++k)
      cp_async8(scr + (s * 3 + k) * 128 + e, p.part + ((size_t)s * p.NPAD + n) * D + 2 * e + 256 * k);
  cp_async_wait_all();
  for (int s = 0; s < nsplit; ++s) {  // in split order: deterministic
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const float2 q = scr[(s * 3 + k) * 128 + e];
      acc[k].x += q.x;
      acc[k].y += q.y;
    }
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    if (nsplit > 0) {
      x[k].x += g[k].x * acc[k].x;
      x[k].y += g[k].y * acc[k].y;
      *reinterpret_cast<float2*>(p.x + (size_t)n * D + 2 * e + 256 * k) = x[k];
    }
    v[2 * k] = x[k].x;
    v[2 * k + 1] = x[k].y;
  }
}

// xn = x * rsqrt(mean(x^2) + 1e-6) * (1 + scale) + shift -> bf16 (mk_ma2.cu:130-158).
__device__ __forceinline__ void row_rms_store(const Params& p, int n, const float v[6], const float* mod, float* red) {
  const int e = threadIdx.x - 64;
  float2 sc[3], sh[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    sc[k] = __ldg(reinterpret_cast<const float2*>(mod + 2 * e + 256 * k));
    sh[k] = __ldg(reinterpret_cast<const float2*>(mod + D + 2 * e + 256 * k));
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 6; ++i) ss += v[i] * v[i];
  ss = epi_sum(ss, red);
  const float r = rsqrtf(ss * (1.0f / D) + kEps);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    __nv_bfloat162 o = __floats2bfloat162_rn(v[2 * k] * r * (1.f + sc[k].x) + sh[k].x,
                                             v[2 * k + 1] * r * (1.f + sc[k].y) + sh[k].y);
    *reinterpret_cast<__nv_bfloat162*>(p.xn + (size_t)n * D + 2 * e + 256 * k) = o;
  }
}

// x += gate * sum_s part[s] (partials already carry the bias), xn = adaRMS(x; mod).
__device__ __forceinline__ void stage_norm(const Params& p, const float* gate, int nsplit, const float* mod, float* red,
                                           float2* scr) {
  for (int n = blockIdx.x; n < p.NT; n += gridDim.x) {
    float v[6];
    row_load_residual(p, n, gate, nsplit, v, scr);
    row_rms_store(p, n, v, mod, red);
  }
}

// x = W_ain x_t + b_ain (mk_ma2.cu:259-268), then the first adaRMS of block 0 of `step`.
__device__ void embed_norm_token(const Params& p, int n, int step, const float* xt, float* red) {
  const int e = threadIdx.x - 64;
  float v[6];
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    const int d = 2 * e + 256 * (i >> 1) + (i & 1);
    float acc = p.b_ain[d];
    const float* w = p.w_ain + (size_t)d * p.AD;
    for (int a = 0; a < p.AD; ++a) acc = fmaf(w[a], xt[a], acc);
    v[i] = acc;
  }
#pragma unroll
  for (int k = 0; k < 3; ++k)
    *reinterpret_cast<float2*>(p.x + (size_t)n * D + 2 * e + 256 * k) = make_float2(v[2 * k], v[2 * k + 1]);
  row_rms_store(p, n, v, mod_ptr(p, step, 0, 0), red);
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

// Final adaRMS (scale, shift), velocity head on the valid action dims, x_t += dt v
// (mk_ma2.cu:558-575), then the next step's embed + first norm.
__device__ __noinline__ void stage_final(const Params& p, int step, float* xf, float* xt_s, float* red) {
  const int e = threadIdx.x - 64, lane = e & 31, w = e >> 5;
  const float* gate = mod_ptr(p, step, p.L - 1, 2) + 2 * D;
  const float* modf = p.mod_final + (size_t)step * 2 * D;
  for (int n = blockIdx.x; n < p.NT; n += gridDim.x) {
    float v[6];
    row_load_residual(p, n, gate, p.split[MAT_DN], v, reinterpret_cast<float2*>(xf + 2048));  // scratch after xf
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 6; ++i) ss += v[i] * v[i];
    ss = epi_sum(ss, red);
    const float r = rsqrtf(ss * (1.0f / D) + kEps);
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const int d = 2 * e + 256 * (i >> 1) + (i & 1);
      xf[d] = v[i] * r * (1.f + modf[d]) + modf[D + d];
    }
    sync_epi();
    for (int a = w; a < p.AD; a += 4) {
      const float* wr = p.w_aout + (size_t)a * D;
      float acc = 0.f;
      for (int d = lane; d < D; d += 32) acc = fmaf(wr[d], xf[d], acc);
      acc = warp_sum(acc);
      if (lane == 0) {
        float nv = p.x_t[(size_t)n * p.AD + a];
        if (a < p.adim) nv += p.dt * (acc + p.b_aout[a]);  // padded action dims are left untouched
        p.x_t[(size_t)n * p.AD + a] = nv;
        xt_s[a] = nv;
      }
    }
    sync_epi();
    if (step + 1 < p.nsteps) embed_norm_token(p, n, step + 1, xt_s, red);
    sync_epi();
  }
}

// ------------------------------------------------------------------ self-attention (warps 2-5)
// Unit = (observation b, head h, group of 8 query tokens): the queries attend to all T action
// tokens of the observation. q, k get a weightless RMS norm over the 96 head dims and half-split
// RoPE (pairs i, i+48) at positions 0..T-1 from the bound tables; scale 1/sqrt(96)
// (mk_ma2.cu:293-384). Every global load of a phase is issued before its first use.
constexpr int kSelfQMax = TMAX;  // query tokens per self-attention unit: Params::self_q (8 or 32)

__device__ __forceinline__ void bf16x8_to_f32(const uint4& raw, float* dst) {
  const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = __bfloat1622float2(b2[q]);
    dst[2 * q] = f.x;
    dst[2 * q + 1] = f.y;
  }
}

__device__ __forceinline__ void stage_self_attn(const Params& p, float* sm) {
  const int e = threadIdx.x - 64, lane = e & 31, wq = e >> 5;
  const int T = p.T;
  const int kSelfQ = p.self_q;
  const int ngroups = (T + kSelfQ - 1) / kSelfQ;
  float* ks = sm;                  // [32][97] keys (normed + rotated)
  float* vs = ks + TMAX * 97;      // [32][96]
  float* qs = vs + TMAX * 96;      // [self_q][97]
  float* ps = qs + kSelfQMax * 97; // [self_q][33]
  float* rc = ps + kSelfQMax * 33; // [T][48] RoPE cos, then [T][48] sin
  const float scale = 0.10206207261596577f;  // 1/sqrt(96)
  const int T48 = T * 48;
  for (int u = blockIdx.x; u < p.B * H * ngroups; u += gridDim.x) {
    const int b = u / (H * ngroups), h = (u / ngroups) % H, g = u % ngroups;
    const int t0 = g * kSelfQ, nq = min(kSelfQ, T - t0);
    // rows: k (T), v (T), q (nq); 12 16-byte pieces per 96-dim row
    const int nrows = 2 * T + nq;
    uint4 raw[9];  // up to 2 x 32 key / value rows + 32 query rows of 12 pieces
#pragma unroll
    for (int it = 0; it < 9; ++it) {
      const int idx = e + it * 128;
      if (idx < nrows * 12) {
        const int row = idx / 12, seg = idx % 12;
        const int sec = row < T ? 1 : (row < 2 * T ? 2 : 0);
        const int t = row < T ? row : (row < 2 * T ? row - T : t0 + row - 2 * T);
        raw[it] = __ldg(reinterpret_cast<const uint4*>(p.qkv + (size_t)(b * T + t) * QKV_ROWS + sec * D + h * HD) + seg);
      }
    }
    for (int i = e; i < T48 / 4; i += 128) {  // RoPE tables into shared memory (loads in flight with the rows')
      reinterpret_cast<float4*>(rc)[i] = __ldg(reinterpret_cast<const float4*>(p.rope_cos) + i);
      reinterpret_cast<float4*>(rc + T48)[i] = __ldg(reinterpret_cast<const float4*>(p.rope_sin) + i);
    }
#pragma unroll
    for (int it = 0; it < 9; ++it) {
      const int idx = e + it * 128;
      if (idx < nrows * 12) {
        const int row = idx / 12, seg = idx % 12;
        float* dst = row < T ? ks + row * 97 : (row < 2 * T ? vs + (row - T) * 96 : qs + (row - 2 * T) * 97);
        bf16x8_to_f32(raw[it], dst + seg * 8);
      }
    }
    sync_epi();
    for (int row = wq; row < T + nq; row += 4) {  // RMS over the head dims: key rows, then query rows
      float* rp = row < T ? ks + row * 97 : qs + (row - T) * 97;
      const float a0 = rp[lane], a1 = rp[lane + 32], a2 = rp[lane + 64];
      const float r = rsqrtf(warp_sum(a0 * a0 + a1 * a1 + a2 * a2) * (1.0f / HD) + kEps);
      rp[lane] = a0 * r;
      rp[lane + 32] = a1 * r;
      rp[lane + 64] = a2 * r;
    }
    sync_epi();
    for (int idx = e; idx < (T + nq) * 48; idx += 128) {  // half-split RoPE
      const int row = idx / 48, i = idx % 48, t = row < T ? row : t0 + row - T;
      float* rp = row < T ? ks + row * 97 : qs + (row - T) * 97;
      const float c = rc[t * 48 + i], sn = rc[T48 + t * 48 + i];
      const float x1 = rp[i], x2 = rp[i + 48];
      rp[i] = x1 * c - x2 * sn;
      rp[i + 48] = x1 * sn + x2 * c;
    }
    sync_epi();
    for (int idx = e; idx < nq * T; idx += 128) {
      const int t = idx / T, j = idx % T;
      float acc = 0.f;
#pragma unroll 8
      for (int d = 0; d < HD; ++d) acc = fmaf(qs[t * 97 + d], ks[j * 97 + d], acc);
      ps[t * 33 + j] = acc * scale;
    }
    sync_epi();
    for (int t = wq; t < nq; t += 4) {  // softmax over the T keys, one warp per query
      const float sc = lane < T ? ps[t * 33 + lane] : -INFINITY;
      const float m = warp_max(sc);
      const float ex = lane < T ? __expf(sc - m) : 0.f;
      const float sum = warp_sum(ex);
      if (lane < T) ps[t * 33 + lane] = ex / sum;
    }
    sync_epi();
    for (int idx = e; idx < nq * (HD / 2); idx += 128) {  // two dims per thread
      const int t = idx / (HD / 2), d = 2 * (idx % (HD / 2));
      float a0 = 0.f, a1 = 0.f;
      for (int j = 0; j < T; ++j) {
        const float pj = ps[t * 33 + j];
        a0 = fmaf(pj, vs[j * 96 + d], a0);
        a1 = fmaf(pj, vs[j * 96 + d + 1], a1);
      }
      *reinterpret_cast<__nv_bfloat162*>(p.sattn + (size_t)(b * T + t0 + t) * D + h * HD + d) =
          __floats2bfloat162_rn(a0, a1);
    }
    sync_epi();
  }
}

constexpr float kXScale2 = 0.10206207261596577f * kLog2e;  // 1/sqrt(96), log2 units

// ------------------------------------------------------------------ self-attention (tcgen05)
// Unit = (observation b, head h): all T (<= 32) action tokens attend to each other. The epilogue
// warps stage the operands in the work area: warp of lane quadrant 0 the Q rows (token t = lane;
// weightless RMS over the 96 head dims, then half-split RoPE of pairs (i, i + 48) at position t,
// mk_ma2.cu:293-384), quadrant 1 the K rows the same way, quadrant 2 V transposed (V^T[d][t]);
// all as 128-byte-swizzled K-major atoms. S = Q K^T (M 128, N 32, K 128: dims 96..127 zero) ->
// softmax of the T rows on quadrant 0 (scale 1/sqrt(96)) -> P -> O = P V (M 128, N 96, K 32) ->
// the T normalised rows straight into sattn (one key chunk: no merge).
// Work area: Q [0, 32 KB) | K [32, 40 KB) | V^T [40, 52 KB) | P [52 KB, ...): the MMAs read 128
// rows of P, of which only the first 32 (4 KB) are written; the rest lie in the epilogue staging
// area that follows the 64 KB work area and feed result rows that are never read.
constexpr int kSQOff = 0, kSKOff = 32 * 1024, kSVOff = 40 * 1024, kSPOff = 52 * 1024;

// 96 floats -> bf16 row `r` of a 2-atom K-major tile with 128-byte swizzle (dims 96..127 zero);
// the atoms lie `atom_bytes` apart (16 KB for 128-row atoms; less when only the first rows are
// stored and the MMA's other rows may read anything).
__device__ __forceinline__ void store_row_sw128(uint8_t* tile, int r, int atom_bytes, const float* x) {
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    uint8_t* row = tile + a * atom_bytes + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      uint32_t w4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int d = a * 64 + ch * 8 + 2 * k;
        __nv_bfloat162 b2 = __floats2bfloat162_rn(d < 96 ? x[d] : 0.f, d + 1 < 96 ? x[d + 1] : 0.f);
        w4[k] = *reinterpret_cast<uint32_t*>(&b2);
      }
      *reinterpret_cast<uint4*>(row + ((ch ^ (r & 7)) << 4)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
  }
}

// Cross-attention query row of token r, head h: the sum of the cross-q GEMM's K-split partials,
// weightless RMS over the 96 head dims (mk_ma2.cu:293-384); zeros for r >= T.
__device__ __forceinline__ void cross_q_row(const Params& p, int b, int h, int r, float* q) {
  if (r >= p.T) {
#pragma unroll
    for (int k = 0; k < 96; ++k) q[k] = 0.f;
    return;
  }
  const float4* src = reinterpret_cast<const float4*>(p.part + (size_t)(b * p.T + r) * D + h * HD);
#pragma unroll
  for (int k = 0; k < 24; ++k) {
    const float4 v = __ldcg(src + k);
    q[4 * k] = v.x; q[4 * k + 1] = v.y; q[4 * k + 2] = v.z; q[4 * k + 3] = v.w;
  }
#pragma unroll 1
  for (int sp = 1; sp < p.split[MAT_CQ]; ++sp) {
    const float4* s2 = reinterpret_cast<const float4*>(p.part + ((size_t)sp * p.NPAD + b * p.T + r) * D + h * HD);
#pragma unroll
    for (int k = 0; k < 24; ++k) {
      const float4 v = __ldcg(s2 + k);
      q[4 * k] += v.x; q[4 * k + 1] += v.y; q[4 * k + 2] += v.z; q[4 * k + 3] += v.w;
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 96; ++k) ss += q[k] * q[k];
  const float rn = rsqrtf(ss * (1.0f / HD) + kEps);
#pragma unroll
  for (int k = 0; k < 96; ++k) q[k] *= rn;
}

// Row `t` (96 bf16 from qkv) -> RMS -> optional RoPE -> bf16 into a 2-atom K-major tile row `r`
// (dims 96..127 zero). `atom_rows`: rows per atom (128 for Q, 32 for K).
__device__ __forceinline__ void self_stage_row(const __nv_bfloat16* src, const float* cs, const float* sn,
                                               uint8_t* tile, int r, int atom_rows) {
  float x[96];
#pragma unroll
  for (int k = 0; k < 12; ++k) bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(src) + k), x + 8 * k);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 96; ++k) ss += x[k] * x[k];
  const float rn = rsqrtf(ss * (1.0f / HD) + kEps);
#pragma unroll
  for (int i = 0; i < 48; ++i) {
    const float x1 = x[i] * rn, x2 = x[i + 48] * rn;
    x[i] = x1 * cs[i] - x2 * sn[i];
    x[i + 48] = x1 * sn[i] + x2 * cs[i];
  }
  store_row_sw128(tile, r, atom_rows * 128, x);
}

__device__ __forceinline__ bool mma_self(const Params& p, const Ctx& c, MmaState& st_shared) {
  Bars* const br = c.bars;
  const uint32_t tmem = c.tmem;
  uint8_t* const work = c.work;
  int* const err = p.err;
  MmaState st = st_shared;
  const int nunits = p.B * H;
  for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
    const uint32_t ph = st.nu & 1;
    if (!mbar_wait(&br->q_full, ph, err, KERR_ATTN)) return false;  // Q, K, V^T staged
    tc_fence_after();
    if (leader()) {
      const uint64_t dq = sdesc_sw128(work + kSQOff), dk = sdesc_sw128(work + kSKOff);
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int s4 = 0; s4 < 4; ++s4)
          tc_mma_bf16(tmem, dq + (uint64_t)((a * kAtomBytes) >> 4) + 2 * s4, dk + (uint64_t)((a * 32 * 128) >> 4) + 2 * s4,
                      idesc_bf16(128, 32), (a | s4) != 0);
      tc_commit(&br->s_full);
    }
    __syncwarp();
    if (!mbar_wait(&br->p_full, ph, err, KERR_ATTN)) return false;
    tc_fence_after();
    if (leader()) {
      const uint64_t dp = sdesc_sw128(work + kSPOff), dv = sdesc_sw128(work + kSVOff);
#pragma unroll
      for (int s4 = 0; s4 < 2; ++s4) tc_mma_bf16(tmem + 128, dp + 2 * s4, dv + 2 * s4, idesc_bf16(128, 96), s4 != 0);
      tc_commit(&br->o_full);
    }
    __syncwarp();
    ++st.nu;
  }
  if (leader()) st_shared = st;
  __syncwarp();
  return true;
}

__device__ __forceinline__ uint32_t epi_self(const Params& p, const Ctx& c, uint32_t nu) {
  Bars* const br = c.bars;
  const uint32_t tmem = c.tmem;
  uint8_t* const work = c.work;
  int* const err = p.err;
  const int T = p.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3;
  const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
  const int nunits = p.B * H;
  for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
    const int b = u / H, h = u % H;
    const uint32_t ph = nu & 1;
    // stage the operands (the previous unit's O has been drained: its MMAs are done)
    if (lane < T && qd < 2) {
      const int sec = qd == 0 ? 0 : 1;  // q | k section of the qkv row
      self_stage_row(p.qkv + (size_t)(b * T + lane) * QKV_ROWS + sec * D + h * HD, p.rope_cos + lane * 48,
                     p.rope_sin + lane * 48, work + (qd == 0 ? kSQOff : kSKOff), lane, qd == 0 ? 128 : 32);
    } else if (qd < 2) {  // rows of missing tokens: zero (they meet valid rows as keys)
      for (int a = 0; a < 2; ++a) {
        uint8_t* row = work + (qd == 0 ? kSQOff : kSKOff) + a * (qd == 0 ? 128 : 32) * 128 + (lane >> 3) * 1024 + (lane & 7) * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) *reinterpret_cast<uint4*>(row + (ch << 4)) = make_uint4(0, 0, 0, 0);
      }
    } else if (qd == 2) {  // V^T[d][t] for token t = lane: 96 two-byte stores into the swizzled rows
      const unsigned short* src = reinterpret_cast<const unsigned short*>(p.qkv + (size_t)(b * T + lane) * QKV_ROWS + 2 * D + h * HD);
      const int t = lane, chunk = t >> 3;
      uint8_t* vt = work + kSVOff;
#pragma unroll 4
      for (int d = 0; d < 96; ++d) {
        const unsigned short v = lane < T ? __ldg(src + d) : (unsigned short)0;
        *reinterpret_cast<unsigned short*>(vt + (d >> 3) * 1024 + (d & 7) * 128 + ((chunk ^ (d & 7)) << 4) + (t & 7) * 2) = v;
      }
    }
    fence_proxy_async_shared();
    mbar_arrive(&br->q_full);
    if (qd == 0) {  // softmax of the T rows (row = lane), P into the work area
      if (!mbar_wait(&br->s_full, ph, err, KERR_ATTN)) return nu;
      tc_fence_after();
      float v[32];
      tmem_ld16(tmem + lane_addr, v);
      tmem_ld16(tmem + lane_addr + 16, v + 16);
      tc_wait_ld();
      float m = -INFINITY;
#pragma unroll
      for (int k = 0; k < 32; ++k)
        if (k < T) m = fmaxf(m, v[k]);
      m *= kXScale2;
      float sum = 0.f;
      uint32_t pk[16];
#pragma unroll
      for (int k = 0; k < 32; k += 2) {
        const float p0 = k < T ? fast_exp2(fmaf(v[k], kXScale2, -m)) : 0.f;
        const float p1 = k + 1 < T ? fast_exp2(fmaf(v[k + 1], kXScale2, -m)) : 0.f;
        __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
        sum += __low2float(b2) + __high2float(b2);
        pk[k >> 1] = *reinterpret_cast<uint32_t*>(&b2);
      }
      uint8_t* prow = work + kSPOff + (lane >> 3) * 1024 + (lane & 7) * 128;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(prow + ((q ^ (lane & 7)) << 4)) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      fence_proxy_async_shared();
      tc_fence_before();
      mbar_arrive(&br->p_full);
      if (!mbar_wait(&br->o_full, ph, err, KERR_ATTN)) return nu;
      tc_fence_after();
      const float inv = sum > 0.f ? 1.f / sum : 0.f;
#pragma unroll 1
      for (int cc = 0; cc < HD; cc += 32) {
        float o[32];
        tmem_ld16(tmem + lane_addr + 128 + cc, o);
        tmem_ld16(tmem + lane_addr + 128 + cc + 16, o + 16);
        tc_wait_ld();
        if (lane < T) {
#pragma unroll
          for (int k = 0; k < 32; k += 8) {
            uint32_t w4[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              __nv_bfloat162 b2 = __floats2bfloat162_rn(o[k + 2 * q] * inv, o[k + 2 * q + 1] * inv);
              w4[q] = *reinterpret_cast<uint32_t*>(&b2);
            }
            *reinterpret_cast<uint4*>(p.sattn + (size_t)(b * T + lane) * D + h * HD + cc + k) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
        }
      }
      tc_fence_before();
    } else {  // the others: p_full counts all 128 epilogue threads; then wait for the unit's MMAs
      mbar_arrive(&br->p_full);
      if (!mbar_wait(&br->o_full, ph, err, KERR_ATTN)) return nu;
    }
    sync_epi();  // quadrant 0 has drained O before anyone restages the operands
    ++nu;
  }
  return nu;
}

// ------------------------------------------------------------------ cross-attention (tcgen05)
// Unit = (observation b, head h, context chunk c of 128 keys); 8 heads with their own K / V (MHA).
// Per unit, in the 64 KB work area:
//   epilogue warps  Q tile [0, 32 KB): row t = the RMS-normalised cross query of token t (the
//                   K-split partials of the cross-q projection summed in split order, bias on split
//                   0, mk_ma2.cu:398-422), dims 96..127 and rows >= T zero; 2 atoms of 64 dims.
//   MMA lane        K tile [32, 64 KB) by TMA: 128 keys x dims [96 h, 96 h + 128) (the last 32 belong
//                   to the next head and meet Q's zero dims); S = Q K^T (M 128, N 128, K 128) into
//                   TMEM columns 0..127.
//   epilogue warps  softmax of the rows (scale 1/sqrt(96), log2 units) -> P (bf16) into the K area.
//   MMA lane        V^T tile (96 dims x 128 keys, 2 atoms) by TMA into the Q area once S is done;
//                   O = P V (M 128, N 96, K 128) into TMEM columns 128..223.
//   epilogue warps  normalised O rows and (max, sum) of the T valid rows -> opart / oml, merged per
//                   (token, head) by stage_merge.
// q_full, s_full, p_full and o_full complete once per unit of this stage and of the self-attention
// stage (phase = all units so far & 1); k_full, kv_free and v_full once per cross unit only.
constexpr int kXQOff = 0, kXKOff = 32 * 1024;

__device__ __forceinline__ bool mma_cross(const Params& p, const Ctx& c, MmaState& st_shared, int l) {
  const int nunits = c.acnt;
  const AttnUnit* const units = c.au;
  Bars* const br = c.bars;
  const uint32_t tmem = c.tmem;
  uint8_t* const work = c.work;
  int* const err = p.err;
  const CUtensorMap* const maps = p.maps;
  const int L = p.L, LKPAD = p.LKPAD;
  MmaState st = st_shared;
  const uint64_t pol = policy_evict_last();
  for (int u = 0; u < nunits; ++u) {
    const AttnUnit au = units[u];
    const uint32_t ph = st.nu & 1;   // barriers shared with the self-attention units
    const uint32_t phx = st.nq & 1;  // k_full, kv_free, v_full: completed by cross units only
    const int krow = (au.b * L + l) * LKPAD + au.chunk * KC;
    // K (the previous unit's P V has finished reading P from this area: o_full was waited by the
    // epilogue before it built this unit's Q, which we wait for next)
    if (!mbar_wait(&br->q_full, ph, err, KERR_ATTN)) return false;  // Q built, previous unit drained
    FA_ONE(mbar_expect_tx(&br->k_full, 2 * kAtomBytes));
    FA_ONE(tma_load_2d(work + kXKOff, &maps[MAP_KCTX], &br->k_full, 96 * au.hp, krow, pol));
    FA_ONE(tma_load_2d(work + kXKOff + kAtomBytes, &maps[MAP_KCTX], &br->k_full, 96 * au.hp + 64, krow, pol));
    if (!mbar_wait(&br->k_full, phx, err, KERR_ATTN)) return false;
    tc_fence_after();
    if (leader()) {
      const uint32_t id_s = idesc_bf16(128, 128);
      const uint64_t dq0 = sdesc_sw128(work + kXQOff), dk0 = sdesc_sw128(work + kXKOff);
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int s4 = 0; s4 < 4; ++s4)
          tc_mma_bf16(tmem, dq0 + (uint64_t)((a * kAtomBytes) >> 4) + 2 * s4, dk0 + (uint64_t)((a * kAtomBytes) >> 4) + 2 * s4,
                      id_s, (a | s4) != 0);
      tc_commit(&br->s_full);
      tc_commit(&br->kv_free);
    }
    __syncwarp();
    if (!mbar_wait(&br->kv_free, phx, err, KERR_ATTN)) return false;  // S done: Q area free for V
    FA_ONE(mbar_expect_tx(&br->v_full, 2 * 96 * 128));
    FA_ONE(tma_load_3d(work + kXQOff, &maps[MAP_VTCTX], &br->v_full, 0, (au.b * L + l) * D + 96 * au.hp, au.chunk * 2, pol));
    if (!mbar_wait(&br->v_full, phx, err, KERR_ATTN)) return false;
    if (!mbar_wait(&br->p_full, ph, err, KERR_ATTN)) return false;
    tc_fence_after();
    if (leader()) {
      const uint32_t id_o = idesc_bf16(128, 96);
      const uint64_t dp0 = sdesc_sw128(work + kXKOff), dv0 = sdesc_sw128(work + kXQOff);
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
#pragma unroll
        for (int s4 = 0; s4 < 4; ++s4)
          tc_mma_bf16(tmem + 128, dp0 + (uint64_t)((kk * kAtomBytes) >> 4) + 2 * s4,
                      dv0 + (uint64_t)((kk * 96 * 128) >> 4) + 2 * s4, id_o, (kk | s4) != 0);
      tc_commit(&br->o_full);
    }
    __syncwarp();
    ++st.nu;
    ++st.nq;
  }
  if (leader()) st_shared = st;
  __syncwarp();
  return true;
}

// Epilogue side of the tcgen05 cross-attention; `nu` counts this CTA's units over the launch.
__device__ __forceinline__ uint32_t epi_cross(const Params& p, const Ctx& c, uint32_t nu) {
  const int nunits = c.acnt;
  const AttnUnit* const units = c.au;
  Bars* const br = c.bars;
  const uint32_t tmem = c.tmem;
  uint8_t* const work = c.work;
  int* const err = p.err;
  const int T = p.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3;
  const int r = qd * 32 + lane;  // TMEM lane = query row = token
  const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
  for (int u = 0; u < nunits; ++u) {
    const AttnUnit au = units[u];
    const uint32_t ph = nu & 1;
    const int b = au.b, h = au.hp;
    // the previous unit's P V has run (its O was drained below): the Q area is free again
    {  // Q row r: K-split partials summed, RMS, bf16 into the 128-row Q tile
      float q[96];
      cross_q_row(p, b, h, r, q);
      store_row_sw128(work + kXQOff, r, kAtomBytes, q);
    }
    fence_proxy_async_shared();
    mbar_arrive(&br->q_full);
    // softmax of S row r over the chunk's valid keys -> P into the K area
    const int nvalid = min(KC, p.ctx_len[b] - au.chunk * KC);
    if (!mbar_wait(&br->s_full, ph, err, KERR_ATTN)) return nu;
    tc_fence_after();
    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
    for (int cc = 0; cc < KC; cc += 32) {
      float v[32];
      tmem_ld16(tmem + lane_addr + cc, v);
      tmem_ld16(tmem + lane_addr + cc + 16, v + 16);
      tc_wait_ld();
#pragma unroll
      for (int k = 0; k < 32; ++k)
        if (cc + k < nvalid) m4[k & 3] = fmaxf(m4[k & 3], v[k]);
    }
    const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * kXScale2;
    float s4[4] = {0.f, 0.f, 0.f, 0.f};
    uint8_t* prow = work + kXKOff + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll 1
    for (int cc = 0; cc < KC; cc += 32) {
      float v[32];
      tmem_ld16(tmem + lane_addr + cc, v);
      tmem_ld16(tmem + lane_addr + cc + 16, v + 16);
      tc_wait_ld();
      uint32_t pk[16];
#pragma unroll
      for (int k = 0; k < 32; k += 2) {
        const float p0 = cc + k < nvalid ? fast_exp2(fmaf(v[k], kXScale2, -mx)) : 0.f;
        const float p1 = cc + k + 1 < nvalid ? fast_exp2(fmaf(v[k + 1], kXScale2, -mx)) : 0.f;
        __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
        s4[(k >> 1) & 3] += __low2float(b2) + __high2float(b2);
        pk[k >> 1] = *reinterpret_cast<uint32_t*>(&b2);
      }
      uint8_t* base = prow + (cc >> 6) * kAtomBytes;
      const int ch0 = (cc & 63) >> 3;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(base + (((ch0 + q) ^ (r & 7)) << 4)) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    }
    const float sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
    fence_proxy_async_shared();
    tc_fence_before();
    mbar_arrive(&br->p_full);
    // normalised O row r and (max, sum) of the valid rows
    if (!mbar_wait(&br->o_full, ph, err, KERR_ATTN)) return nu;
    tc_fence_after();
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    const size_t slot = ((size_t)(b * H + h) * MAX_CH + au.chunk) * TMAX + r;
#pragma unroll 1
    for (int cc = 0; cc < HD; cc += 32) {
      float v[32];
      tmem_ld16(tmem + lane_addr + 128 + cc, v);
      tmem_ld16(tmem + lane_addr + 128 + cc + 16, v + 16);
      tc_wait_ld();
      if (r < T) {
#pragma unroll
        for (int k = 0; k < 32; k += 8) {
          uint32_t w4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(v[k + 2 * q] * inv, v[k + 2 * q + 1] * inv);
            w4[q] = *reinterpret_cast<uint32_t*>(&b2);
          }
          *reinterpret_cast<uint4*>(p.opart + slot * HD + cc + k) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
    }
    if (r < T) *reinterpret_cast<float2*>(p.oml + slot * 2) = make_float2(nvalid > 0 ? mx : -INFINITY, sum);
    tc_fence_before();
    ++nu;
  }
  return nu;
}

// ------------------------------------------------------------------ cross-attention, whole units
// Unit = (observation b, head h) over all of b's 128-key context chunks, for batches that give
// every SM such a unit: Q is built once per unit, the chunks run as an online softmax (running
// max and sum per query row; the un-normalised O of each chunk is rescaled into registers), and
// the normalised rows go straight to cattn: no per-chunk partials, no merge stage.
// Only the T <= 32 query rows are real, so Q and P keep just rows 0..31 of their two 64-dim
// atoms (atoms 4 KB apart); the MMA's rows 32..127 read whatever follows and produce S / O rows
// that are never read. Work area (64 KB + the 16 KB staging area that follows it):
//   Q [0, 8 KB) | P0 [8, 16 KB) | P1 [16, 24 KB) | K [24, 56 KB) | V^T [56, 80 KB)
// TMEM: S of chunk n in columns (n & 1) * 128, its O in 256 + (n & 1) * 128.
// The MMA lane computes S of chunk c + 1 before P V of chunk c, so the softmax warp finds the next
// S ready; K of chunk c + 2 loads once S of c + 1 is done, V of chunk c + 1 once P V of c is done.
constexpr int kWQOff = 0, kWPOff = 8 * 1024, kWKOff = 24 * 1024, kWVOff = 56 * 1024, kWRowAtom = 4096;

__device__ __forceinline__ bool mma_cross_whole(const Params& p, const Ctx& c, MmaState& st_shared, int l) {
  Bars* const br = c.bars;
  const uint32_t tmem = c.tmem;
  uint8_t* const work = c.work;
  int* const err = p.err;
  const CUtensorMap* const maps = p.maps;
  const int L = p.L, LKPAD = p.LKPAD;
  MmaState st = st_shared;
  const uint64_t pol = policy_evict_last();
  const uint32_t id_s = idesc_bf16(128, 128), id_o = idesc_bf16(128, 96);
  for (int u = 0; u < c.acnt; ++u) {
    const AttnUnit au = c.au[u];
    const int nch = (p.ctx_len[au.b] + KC - 1) / KC;
    const int krow0 = (au.b * L + l) * LKPAD, vrow = (au.b * L + l) * D + 96 * au.hp;
    const uint32_t n0 = st.xc;
    auto load_k = [&](int ch) {
      FA_ONE(mbar_expect_tx(&br->k_full, 2 * kAtomBytes));
      FA_ONE(tma_load_2d(work + kWKOff, &maps[MAP_KCTX], &br->k_full, 96 * au.hp, krow0 + ch * KC, pol));
      FA_ONE(tma_load_2d(work + kWKOff + kAtomBytes, &maps[MAP_KCTX], &br->k_full, 96 * au.hp + 64, krow0 + ch * KC, pol));
    };
    auto load_v = [&](int ch) {
      FA_ONE(mbar_expect_tx(&br->v_full, 2 * 96 * 128));
      FA_ONE(tma_load_3d(work + kWVOff, &maps[MAP_VTCTX], &br->v_full, 0, vrow, ch * 2, pol));
    };
    // S of chunk ch (global chunk index n) into TMEM buffer n & 1; then K of chunk ch + 1
    auto do_s = [&](int ch) -> bool {
      const uint32_t n = n0 + ch, j = n & 1;
      if (!mbar_wait(&br->k_full, n & 1, err, KERR_ATTN)) return false;
      if (!mbar_wait(&br->xs_free[j], ((n >> 1) & 1) ^ 1, err, KERR_ATTN)) return false;
      tc_fence_after();
      if (leader()) {
        const uint64_t dq = sdesc_sw128(work + kWQOff), dk = sdesc_sw128(work + kWKOff);
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
          for (int s4 = 0; s4 < 4; ++s4)
            tc_mma_bf16(tmem + j * 128, dq + (uint64_t)((a * kWRowAtom) >> 4) + 2 * s4,
                        dk + (uint64_t)((a * kAtomBytes) >> 4) + 2 * s4, id_s, (a | s4) != 0);
        tc_commit(&br->xs_full[j]);
        tc_commit(&br->kv_free);
      }
      __syncwarp();
      if (!mbar_wait(&br->kv_free, n & 1, err, KERR_ATTN)) return false;  // K area free
      if (ch + 1 < nch) load_k(ch + 1);
      return true;
    };
    // K and V of the first chunk: both areas are free (the previous unit's last S and P V were
    // waited for below)
    load_k(0);
    load_v(0);
    if (!mbar_wait(&br->xq_full, st.xu & 1, err, KERR_ATTN)) return false;
    if (!do_s(0)) return false;
    for (int ch = 0; ch < nch; ++ch) {
      if (ch + 1 < nch && !do_s(ch + 1)) return false;
      const uint32_t n = n0 + ch, j = n & 1;
      if (!mbar_wait(&br->v_full, n & 1, err, KERR_ATTN)) return false;
      if (!mbar_wait(&br->xp_full[j], (n >> 1) & 1, err, KERR_ATTN)) return false;
      if (!mbar_wait(&br->xo_free[j], ((n >> 1) & 1) ^ 1, err, KERR_ATTN)) return false;
      tc_fence_after();
      if (leader()) {
        const uint64_t dp = sdesc_sw128(work + kWPOff + j * 2 * kWRowAtom), dv = sdesc_sw128(work + kWVOff);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
#pragma unroll
          for (int s4 = 0; s4 < 4; ++s4)
            tc_mma_bf16(tmem + 256 + j * 128, dp + (uint64_t)((kk * kWRowAtom) >> 4) + 2 * s4,
                        dv + (uint64_t)((kk * 96 * 128) >> 4) + 2 * s4, id_o, (kk | s4) != 0);
        tc_commit(&br->xo_full[j]);
        tc_commit(&br->v_free);
      }
      __syncwarp();
      if (!mbar_wait(&br->v_free, n & 1, err, KERR_ATTN)) return false;  // V area free
      if (ch + 1 < nch) load_v(ch + 1);
    }
    st.xc = n0 + nch;
    ++st.xu;
  }
  if (leader()) st_shared = st;
  __syncwarp();
  return true;
}

// Epilogue side of the whole-unit cross-attention: the warp of TMEM lane quadrant 0 (query row =
// lane) alone; `xu` / `xc` count this CTA's units / chunks over the launch.
__device__ __forceinline__ void epi_cross_whole(const Params& p, const Ctx& c, uint32_t& xu, uint32_t& xc) {
  Bars* const br = c.bars;
  const uint32_t tmem = c.tmem;
  uint8_t* const work = c.work;
  int* const err = p.err;
  const int T = p.T, lane = threadIdx.x & 31;
  for (int u = 0; u < c.acnt; ++u) {
    const AttnUnit au = c.au[u];
    const int b = au.b, h = au.hp;
    const int len = p.ctx_len[b], nch = (len + KC - 1) / KC;
    {  // Q: the previous unit's S products have all been waited for below
      float q[96];
      cross_q_row(p, b, h, lane, q);
      store_row_sw128(work + kWQOff, lane, kWRowAtom, q);
    }
    fence_proxy_async_shared();
    mbar_arrive(&br->xq_full);
    float acc[96];
#pragma unroll
    for (int k = 0; k < 96; ++k) acc[k] = 0.f;
    float m_run = -INFINITY, l_run = 0.f, m_acc = -INFINITY, m_last = -INFINITY;
    // O of chunk n (computed against running max m_n) folded into acc
    auto fold = [&](uint32_t n, float m_n) -> bool {
      const uint32_t j = n & 1;
      if (!mbar_wait(&br->xo_full[j], (n >> 1) & 1, err, KERR_ATTN)) return false;
      tc_fence_after();
      const float alpha = fast_exp2(m_acc - m_n);
#pragma unroll
      for (int cc = 0; cc < HD; cc += 32) {
        float o[32];
        tmem_ld16(tmem + 256 + j * 128 + cc, o);
        tmem_ld16(tmem + 256 + j * 128 + cc + 16, o + 16);
        tc_wait_ld();
#pragma unroll
        for (int k = 0; k < 32; ++k) acc[cc + k] = fmaf(acc[cc + k], alpha, o[k]);
      }
      m_acc = m_n;
      tc_fence_before();
      mbar_arrive(&br->xo_free[j]);
      return true;
    };
    for (int ch = 0; ch < nch; ++ch) {
      const uint32_t n = xc + ch, j = n & 1;
      const int nvalid = min(KC, len - ch * KC);
      if (!mbar_wait(&br->xs_full[j], (n >> 1) & 1, err, KERR_ATTN)) return;
      tc_fence_after();
      const uint32_t scol = tmem + j * 128;
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
      for (int cc = 0; cc < KC; cc += 32) {
        float v[32];
        tmem_ld16(scol + cc, v);
        tmem_ld16(scol + cc + 16, v + 16);
        tc_wait_ld();
#pragma unroll
        for (int k = 0; k < 32; ++k)
          if (cc + k < nvalid) m4[k & 3] = fmaxf(m4[k & 3], v[k]);
      }
      const float m_new = fmaxf(m_run, fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * kXScale2);
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
      uint8_t* prow = work + kWPOff + j * 2 * kWRowAtom + (lane >> 3) * 1024 + (lane & 7) * 128;
#pragma unroll 1
      for (int cc = 0; cc < KC; cc += 32) {
        float v[32];
        tmem_ld16(scol + cc, v);
        tmem_ld16(scol + cc + 16, v + 16);
        tc_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          const float p0 = cc + k < nvalid ? fast_exp2(fmaf(v[k], kXScale2, -m_new)) : 0.f;
          const float p1 = cc + k + 1 < nvalid ? fast_exp2(fmaf(v[k + 1], kXScale2, -m_new)) : 0.f;
          __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
          s4[(k >> 1) & 3] += __low2float(b2) + __high2float(b2);
          pk[k >> 1] = *reinterpret_cast<uint32_t*>(&b2);
        }
        uint8_t* base = prow + (cc >> 6) * kWRowAtom;
        const int ch0 = (cc & 63) >> 3;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(base + (((ch0 + q) ^ (lane & 7)) << 4)) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
      tc_fence_before();
      mbar_arrive(&br->xs_free[j]);
      l_run = fmaf(l_run, fast_exp2(m_run - m_new), (s4[0] + s4[1]) + (s4[2] + s4[3]));
      m_run = m_new;
      fence_proxy_async_shared();
      mbar_arrive(&br->xp_full[j]);
      if (ch > 0 && !fold(n - 1, m_last)) return;
      m_last = m_new;
    }
    if (!fold(xc + nch - 1, m_last)) return;
    xc += nch;
    ++xu;
    if (lane < T) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(p.cattn + (size_t)(b * T + lane) * D + h * HD);
#pragma unroll
      for (int k = 0; k < 96; k += 8) {
        uint32_t w4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          __nv_bfloat162 b2 = __floats2bfloat162_rn(acc[k + 2 * q] * inv, acc[k + 2 * q + 1] * inv);
          w4[q] = *reinterpret_cast<uint32_t*>(&b2);
        }
        dst[k / 8] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
    }
  }
}

// Merge of the context chunks per (token, head): out = sum_c w_c O_c / sum_c w_c,
// w_c = 2^(m_c - M) l_c. One warp per (token, head); lane j holds chunks j, j + 32, ...
__device__ __forceinline__ void stage_merge(const Params& p) {
  const int e = threadIdx.x - 64, lane = e & 31, wq = e >> 5;
  constexpr int kPer = MAX_CH / 32;
  for (int item = blockIdx.x * 4 + wq; item < p.NT * H; item += gridDim.x * 4) {
    const int n = item / H, h = item % H;
    const int b = tok_b(p, n), t = n - b * p.T;
    const int nch = (p.ctx_len[b] + KC - 1) / KC;
    const size_t base = (size_t)(b * H + h) * MAX_CH;
    // the first 16 chunks' rows are loaded together with the (max, sum) pairs: one round trip
    // per item for contexts up to 512 tokens
    unsigned short rv[16][3];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const unsigned short* src = reinterpret_cast<const unsigned short*>(p.opart) + ((base + j) * TMAX + t) * HD + lane;
#pragma unroll
      for (int k = 0; k < 3; ++k) rv[j][k] = j < nch ? __ldcg(src + 32 * k) : (unsigned short)0;
    }
    float2 ml[kPer];
    float mloc = -INFINITY;
#pragma unroll
    for (int g = 0; g < kPer; ++g) {
      const int cidx = lane + 32 * g;
      ml[g] = cidx < nch ? __ldcg(reinterpret_cast<const float2*>(p.oml + ((base + cidx) * TMAX + t) * 2))
                         : make_float2(-INFINITY, 0.f);
      mloc = fmaxf(mloc, ml[g].x);
    }
    const float M = warp_max(mloc);
    float w_own[kPer], wloc = 0.f;
#pragma unroll
    for (int g = 0; g < kPer; ++g) {
      w_own[g] = ml[g].y > 0.f ? fast_exp2(ml[g].x - M) * ml[g].y : 0.f;
      wloc += w_own[g];
    }
    const float wsum = warp_sum(wloc);
    float acc[3] = {0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float wgt = __shfl_sync(0xffffffffu, w_own[0], j);
#pragma unroll
      for (int k = 0; k < 3; ++k) acc[k] += wgt * __bfloat162float(__ushort_as_bfloat16(rv[j][k]));
    }
#pragma unroll
    for (int g = 0; g < kPer; ++g) {
      if (32 * g >= nch) break;
#pragma unroll 8
      for (int j = g == 0 ? 16 : 0; j < 32; ++j) {
        const int cidx = 32 * g + j;
        const float wgt = __shfl_sync(0xffffffffu, w_own[g], j);
        if (cidx < nch) {
          const __nv_bfloat16* src = p.opart + ((base + cidx) * TMAX + t) * HD;
#pragma unroll
          for (int k = 0; k < 3; ++k) acc[k] += wgt * __bfloat162float(__ldcg(src + lane + 32 * k));
        }
      }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
    for (int k = 0; k < 3; ++k) p.cattn[(size_t)n * D + h * HD + lane + 32 * k] = __float2bfloat16(acc[k] * inv);
  }
}

// ------------------------------------------------------------------ GEMM epilogues and model traits
struct Ma2Epi {
  int NT, NPAD;
  uint8_t* stage;
  __nv_bfloat16* qkv;
  __nv_bfloat16* hbuf;
  float* part;
  const float* bias[NUM_MATS];  // this layer's bias of each matrix (gate bias for MAT_GU)
  const float* b_up;            // this layer's up bias
};

__device__ __forceinline__ int mat_rows(int m) { return m == MAT_QKV ? QKV_ROWS : (m == MAT_GU ? 2 * F : D); }

struct Ma2Model {
  using Params = ma2::Params;
  using Epi = Ma2Epi;
  static constexpr int kMats = NUM_MATS;  // QKV, self-out, cross-q, cross-out, gate/up, down
  static constexpr bool kF8 = false;       // bf16 weight stream only
  static constexpr bool kTM = false;       // token-major GEMMs (one tile of <= 64 tokens)
  __device__ static float row_scale(const Params&, int, int, int, int) { return 1.0f; }
  __device__ static int rows(int m) { return mat_rows(m); }
  __device__ static int wmap(int m) { return MAP_W_QKV + m; }
  __device__ static int wmap_half(int m) { return MAP_W_QKV + m; }  // no half-row units here
  __device__ static int act_map(int m) {
    return m == MAT_SO ? MAP_SATTN : m == MAT_CO ? MAP_CATTN : m == MAT_DN ? MAP_H : MAP_XN;
  }
  __device__ static int trace_stage(int m) {
    const int st[NUM_MATS] = {ST_QKV, ST_SO, ST_CQ, ST_CO, ST_GU, ST_DN};
    return st[m];
  }
  __device__ static void epi_load(Epi& e, const Params& p, const Ctx& c, int l) {
    e.NT = p.NT; e.NPAD = p.NPAD; e.stage = c.stage; e.qkv = p.qkv; e.hbuf = p.hbuf; e.part = p.part;
#pragma unroll
    for (int m = 0; m < NUM_MATS; ++m) e.bias[m] = p.bias[m] + (size_t)l * (m == MAT_GU ? F : (m == MAT_QKV ? QKV_ROWS : D));
    e.b_up = p.b_up + (size_t)l * F;
  }
  __device__ static bool staged(int m, const GemmUnit&) { return m == MAT_QKV || m == MAT_GU; }
  // 16 tokens (nb..nb+15) of accumulator row `row` of unit gu (mk_ma2.cu:224-251 epilogues).
  __device__ static void epi_tile(const Epi& e, const GemmUnit& gu, int m, int qd, int lane, int row, int nb,
                                  int nb0, const float* v) {
    if (m == MAT_QKV) {  // + bias, bf16, staged as [token][128 rows]
      const float bias = e.bias[m][gu.mtile * 128 + row];
      __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(e.stage) + (nb - nb0) * 128 + row;
#pragma unroll
      for (int k = 0; k < 16; ++k) st[k * 128] = __float2bfloat16(v[k] + bias);
    } else if (m == MAT_GU) {  // lanes 0-15 gate rows, 16-31 up rows of one feature: silu(g) * u
      const int f = 64 * gu.mtile + 16 * qd + (lane & 15);
      const float bias = lane < 16 ? e.bias[MAT_GU][f] : e.b_up[f];
      float gu_v[16], up[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) gu_v[k] = v[k] + bias;
#pragma unroll
      for (int k = 0; k < 16; ++k) up[k] = __shfl_xor_sync(0xffffffffu, gu_v[k], 16);
      if (lane < 16) {
        __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(e.stage) + (nb - nb0) * 64 + 16 * qd + lane;
#pragma unroll
        for (int k = 0; k < 16; ++k) st[k * 64] = __float2bfloat16(gu_v[k] / (1.f + __expf(-gu_v[k])) * up[k]);
      }
    } else {  // self-out / cross-q / cross-out / down: fp32 K-split partial, bias carried by split 0
      const float bias = gu.split == 0 ? e.bias[m][gu.mtile * 128 + row] : 0.f;
      float* dst = e.part + ((size_t)gu.split * e.NPAD + nb) * D + gu.mtile * 128 + row;
#pragma unroll
      for (int k = 0; k < 16; ++k) dst[(size_t)k * D] = v[k] + bias;
    }
  }
  // Copies staged rows (tokens) [r0, r1) of the 64-token sub-tile at nb0.
  __device__ static void epi_copy_out(const Epi& e, const GemmUnit& gu, int m, int nb0, int r0, int r1) {
    const int t_ = threadIdx.x - 64;
    if (m == MAT_GU) {  // 64 tokens x 128 B
      for (int it = t_; it < (r1 - r0) * 8; it += 128) {
        const int t = r0 + (it >> 3), seg = it & 7, n = nb0 + t;
        if (n >= e.NT) continue;
        *reinterpret_cast<uint4*>(e.hbuf + (size_t)n * F + 64 * gu.mtile + seg * 8) =
            *reinterpret_cast<const uint4*>(e.stage + t * 128 + seg * 16);
      }
    } else {  // 64 tokens x 256 B into qkv [NPAD][2304]
      __nv_bfloat16* out = e.qkv;
      const int stride = QKV_ROWS;
      for (int it = t_; it < (r1 - r0) * 16; it += 128) {
        const int t = r0 + (it >> 4), seg = it & 15, n = nb0 + t;
        if (n >= e.NT) continue;
        *reinterpret_cast<uint4*>(out + (size_t)n * stride + gu.mtile * 128 + seg * 8) =
            *reinterpret_cast<const uint4*>(e.stage + t * 256 + seg * 16);
      }
    }
  }
};

// Token-major traits (bound batch = one tile of <= 64 tokens): thread = token n, v = 32
// consecutive accumulator columns c0.. = 32 consecutive rows of the unit's 128-row weight tile.
// In the packed gate/up tile, rows 32 q + i (i < 16) are the gate and rows 32 q + 16 + i the up
// projection of feature 64 mtile + 16 q + i (the same packing as the weight-major epilogue).
struct Ma2ModelTM : Ma2Model {
  static constexpr bool kTM = true;
  __device__ static void epi_tm(const Epi& e, const GemmUnit& gu, int m, int n, int c0, const float* v) {
    if (n >= e.NT) return;
    const int r0 = gu.mtile * 128 + c0;
    auto pack = [](float lo, float hi) {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(lo, hi);
      return *reinterpret_cast<uint32_t*>(&b2);
    };
    if (m == MAT_QKV) {  // + bias -> bf16 row n of qkv
      const float* b = e.bias[MAT_QKV] + r0;
      uint4* d = reinterpret_cast<uint4*>(e.qkv + (size_t)n * QKV_ROWS + r0);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        d[k] = make_uint4(pack(v[8 * k] + b[8 * k], v[8 * k + 1] + b[8 * k + 1]), pack(v[8 * k + 2] + b[8 * k + 2], v[8 * k + 3] + b[8 * k + 3]),
                          pack(v[8 * k + 4] + b[8 * k + 4], v[8 * k + 5] + b[8 * k + 5]), pack(v[8 * k + 6] + b[8 * k + 6], v[8 * k + 7] + b[8 * k + 7]));
    } else if (m == MAT_GU) {  // silu(gate + b_gate) * (up + b_up) -> bf16 features f0 .. f0 + 15
      const int f0 = 64 * gu.mtile + 16 * (c0 >> 5);
      float h[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float g = v[i] + e.bias[MAT_GU][f0 + i], u = v[16 + i] + e.b_up[f0 + i];
        h[i] = g / (1.f + __expf(-g)) * u;
      }
      uint4* d = reinterpret_cast<uint4*>(e.hbuf + (size_t)n * F + f0);
      d[0] = make_uint4(pack(h[0], h[1]), pack(h[2], h[3]), pack(h[4], h[5]), pack(h[6], h[7]));
      d[1] = make_uint4(pack(h[8], h[9]), pack(h[10], h[11]), pack(h[12], h[13]), pack(h[14], h[15]));
    } else {  // fp32 K-split partial, bias carried by split 0
      const float* b = e.bias[m] + r0;
      float4* d = reinterpret_cast<float4*>(e.part + ((size_t)gu.split * e.NPAD + n) * D + r0);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float4 o = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
        if (gu.split == 0) { o.x += b[4 * k]; o.y += b[4 * k + 1]; o.z += b[4 * k + 2]; o.w += b[4 * k + 3]; }
        d[k] = o;
      }
    }
  }
};

// ------------------------------------------------------------------ kernel
template <class Model>
__device__ __forceinline__ void ma2_denoise_body(const Params& p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars bars;
  __shared__ uint32_t s_tmem;
  __shared__ float s_red[8];
  __shared__ float s_xt[32];
  __shared__ CtaPlan s_plan;
  __shared__ GemmUnit s_gu[kMaxGU];
  __shared__ AttnUnit s_au[kMaxAU];
  __shared__ Ctx s_c;
  __shared__ MmaState s_st;
  const int warp = threadIdx.x >> 5;
  Ctx& c = s_c;
  if (threadIdx.x == 0) {
    s_plan = p.plans[blockIdx.x];
    g_trp = nullptr;
    s_st.wit = s_st.bload = s_st.bfree = s_st.acc = s_st.nq = s_st.nu = s_st.xu = s_st.xc = s_st.qtm = 0;
    s_st.last_q = -1;
    s_st.k_pre = 0;
  }
  __syncthreads();
  {
    int ng = 0;
    for (int m = 0; m < NUM_MATS; ++m) ng += s_plan.g_cnt[m];
    for (int i = threadIdx.x; i < ng; i += blockDim.x) s_gu[i] = p.gunits[s_plan.g_off[0] + i];
    for (int i = threadIdx.x; i < s_plan.a_cnt; i += blockDim.x) s_au[i] = p.aunits[s_plan.a_off + i];
  }
  if (threadIdx.x == 0) {
    for (int m = 0, off = 0; m < NUM_MATS; ++m) {
      c.gu[m] = s_gu + off;
      c.gcnt[m] = s_plan.g_cnt[m];
      off += s_plan.g_cnt[m];
    }
    c.au = s_au;
    c.acnt = s_plan.a_cnt;
    c.batoms = min(kMaxBAtoms, s_plan.b_bytes / (p.NTILE * 128));
    c.ring_slots = s_plan.ring_slots;
    c.ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    c.work = c.ring + (size_t)c.ring_slots * p.wg * kAtomBytes;
    c.stage = c.work + max(s_plan.b_bytes, kMinWork);
    c.tm_slots = min(4, s_plan.b_bytes / (int)kTmChunkBytes);
    c.bars = &bars;
    for (int i = 0; i < kMaxRing; ++i) { mbar_init(&bars.wfull[i], 1); mbar_init(&bars.wempty[i], 1); }
    mbar_init(&bars.bfull, 1);
    mbar_init(&bars.bempty, 1);
    for (int i = 0; i < 4; ++i) { mbar_init(&bars.sfull[i], 1); mbar_init(&bars.sempty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&bars.acc_full[i], 1); mbar_init(&bars.acc_empty[i], 128); }
    mbar_init(&bars.drain, 1);
    // tcgen05 cross-attention: Q built / K / S / S done / V / P written / O, once per unit
    mbar_init(&bars.q_full, 128); mbar_init(&bars.k_full, 1); mbar_init(&bars.s_full, 1);
    mbar_init(&bars.kv_free, 1); mbar_init(&bars.v_full, 1); mbar_init(&bars.p_full, 128); mbar_init(&bars.o_full, 1);
    mbar_init(&bars.v_free, 1); mbar_init(&bars.xq_full, 32);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.xs_full[i], 1); mbar_init(&bars.xs_free[i], 32); mbar_init(&bars.xp_full[i], 32);
      mbar_init(&bars.xo_full[i], 1); mbar_init(&bars.xo_free[i], 32);
    }
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
    uint32_t ecnt = 0, gen = 0, xnu = 0;  // xnu: attention units done (epilogue warps)
    uint32_t xwu = 0, xwc = 0;             // whole-unit cross-attention: units, key chunks (lane quadrant 0)
    ConvState cs{0, 0};  // FP8 conversion state (unused by this bf16 kernel)
    uint64_t t_prev = globaltimer();
    const bool timing = p.stage_ns != nullptr && blockIdx.x == 0 && threadIdx.x == 32;
    auto mark = [&](int s) {
      if (timing) {
        const uint64_t t = globaltimer();
        p.stage_ns[s] += t - t_prev;
        t_prev = t;
      }
    };
    auto tr = [&](int stage, int step, int l) -> unsigned long long* {
      if (!p.trace || step != p.trace_step || l != p.trace_layer) return nullptr;
      return p.trace + ((size_t)stage * gridDim.x + blockIdx.x) * kTrStride;
    };
    float* vsm = reinterpret_cast<float*>(c.work);  // vector-stage scratch (no TMA in flight there)
    bool ok = true;
    if (is_epi) stage_embed(p, s_xt, s_red);
    ok = grid_barrier(p, gen++, tr(ST_QKV, 0, 0));
    mark(ST_NORM1);
    // One pass of the loop body per stage; every role function has ONE call site (inlined, no
    // ABI calls between stages). Stage order per block: QKV, self-attention, self-out, norm(mca),
    // cross-q, cross-attention, merge, cross-out, norm(mlp), gate/up, down, norm1 | final.
    // (selects instead of arrays: a runtime-indexed array would live in local memory)
    auto gemm_of = [](int s) {
      return s == 0 ? MAT_QKV : s == 2 ? MAT_SO : s == 4 ? MAT_CQ : s == 7 ? MAT_CO : s == 9 ? MAT_GU
           : s == 10 ? MAT_DN : -1;
    };
    auto timed = [](int s) {
      return s == 0 ? ST_QKV : s == 1 ? ST_SELF : s == 2 ? ST_SO : s == 3 ? ST_NORM2 : s == 4 ? ST_CQ
           : s == 5 ? ST_CROSS : s == 6 ? ST_MERGE : s == 7 ? ST_CO : s == 8 ? ST_NORM3 : s == 9 ? ST_GU
           : s == 10 ? ST_DN : ST_NORM1;
    };
#pragma unroll 1
    for (int step = 0; ok && step < p.nsteps; ++step) {
#pragma unroll 1
      for (int l = 0; ok && l < p.L; ++l) {
        const float* m_self = mod_ptr(p, step, l, 0);
        const float* m_cross = mod_ptr(p, step, l, 1);
        const float* m_mlp = mod_ptr(p, step, l, 2);
        const bool last_layer = l + 1 == p.L;
#pragma unroll 1
        for (int s = 0; s < 12; ++s) {
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
            if (p.self_tc) {
              if (is_mma) mma_self(p, c, st);
              if (is_epi) xnu = epi_self(p, c, xnu);
            } else if (is_epi) {
              stage_self_attn(p, vsm);
            }
          } else if (s == 5) {
            if (p.cross_whole) {
              if (is_mma) mma_cross_whole(p, c, st, l);
              if (is_epi && (warp & 3) == 0) epi_cross_whole(p, c, xwu, xwc);
            } else {
              if (is_mma) mma_cross(p, c, st, l);
              if (is_epi) xnu = epi_cross(p, c, xnu);
            }
          } else if (s == 6) {
            if (is_epi && !p.cross_whole) stage_merge(p);
          } else if (s == 3 || s == 8 || !last_layer) {  // norm(mca) | norm(mlp) | next block's norm(msa)
            if (is_epi) {
              const float* gate = (s == 3 ? m_self : s == 8 ? m_cross : m_mlp) + 2 * D;
              const int ns = p.split[s == 3 ? MAT_SO : s == 8 ? MAT_CO : MAT_DN];
              const float* mod = s == 3 ? m_cross : s == 8 ? m_mlp : mod_ptr(p, step, l + 1, 0);
              stage_norm(p, gate, ns, mod, s_red, reinterpret_cast<float2*>(vsm));  // work area idle here
            }
          } else if (is_epi) {
            stage_final(p, step, vsm, s_xt, s_red);
          }
          const int nxt = s < 11 ? timed(s + 1) : ST_QKV;
          const int nstep = s < 11 ? step : (last_layer ? step + 1 : step);
          const int nl = s < 11 ? l : (last_layer ? 0 : l + 1);
          if (!(ok = grid_barrier(p, gen++, tr(nxt == ST_NORM1 && last_layer ? ST_FINAL : nxt, nstep, nl)))) break;
          mark(s == 11 && last_layer ? ST_FINAL : timed(s));
        }
      }
    }
    if (is_mma) {
      FA_ONE(tc_commit(&bars.drain));
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

__global__ void __launch_bounds__(kThreads, 1) ma2_denoise_kernel(const __grid_constant__ Params p) {
  ma2_denoise_body<Ma2Model>(p);
}
__global__ void __launch_bounds__(kThreads, 1) ma2_denoise_kernel_tm(const __grid_constant__ Params p) {
  ma2_denoise_body<Ma2ModelTM>(p);
}

}  // namespace ma2
}  // namespace fa
