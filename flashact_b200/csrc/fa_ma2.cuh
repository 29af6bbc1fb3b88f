// MolmoAct2 action-expert flow megakernel: parameters shared by host and device.
//
// Reference semantics: src/molmoact2/mk_ma2.cu:103-576 (block structure, modulation layout
// [S][L][3][3][768] = (self, cross, mlp) x (scale, shift, gate), mod_final [S][2][768] =
// (scale, shift), dt = +1/N, action-dim mask) and benchmarks/molmoact2/eval_numerics.py:77-133
// (weight packing). Architecture constants are those of the 36-block DiT action expert.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

#include "fa_engine_types.cuh"

namespace fa {
namespace ma2 {

constexpr int D = 768;       // width
constexpr int H = 8;         // heads (self and cross attention, one KV head each)
constexpr int HD = 96;       // head dim
constexpr int F = 3072;      // SiLU-gated MLP hidden
constexpr int QKV_ROWS = 3 * D;
constexpr int MOD = 3 * D;   // scale | shift | gate of one norm
constexpr int TMAX = 32;     // action tokens per observation (padded)
constexpr int KC = 128;      // context keys per cross-attention unit (one 128-key tcgen05 tile)
constexpr int MAX_CH = 32;   // context chunks per observation (context <= 4096 tokens)
constexpr int kMinWork = 64 * 1024;  // every CTA keeps this much work area for the vector stages

enum Mat : int { MAT_QKV = 0, MAT_SO, MAT_CQ, MAT_CO, MAT_GU, MAT_DN, NUM_MATS };
enum Map : int {
  MAP_W_QKV = 0, MAP_W_SO, MAP_W_CQ, MAP_W_CO, MAP_W_GU, MAP_W_DN,  // weights, box {64, 128}
  MAP_XN, MAP_SATTN, MAP_CATTN, MAP_H,                              // activations, 3D boxes
  MAP_KCTX, MAP_VTCTX,  // cross-attention context: K rows (2D, box 64 dims x 128 keys), V^T (3D, 96 dims x 128 keys)
  NUM_MAPS
};
enum Stage : int {
  ST_NORM1 = 0, ST_QKV, ST_SELF, ST_SO, ST_NORM2, ST_CQ, ST_CROSS, ST_MERGE, ST_CO, ST_NORM3, ST_GU, ST_DN,
  ST_FINAL, NUM_STAGES
};

struct Params {
  CUtensorMap maps[NUM_MAPS];
  // geometry
  int L, T, B, NT, NPAD, NTILE, TG, ngroups, nsteps, AD, adim, LKPAD;
  int split[NUM_MATS];  // K-split factor per matrix (1 = full K, epilogue sees the final sum)
  int tg[kMaxMats];  // token tiles per group (one accumulator) of each GEMM matrix
  int self_tc;      // self-attention on tcgen05 (one unit per observation and head)
  int cross_whole;  // cross-attention units cover all context chunks of one (observation, head); no merge
  int self_q;       // query tokens per self-attention unit (8, or 32 = all of an observation's tokens)
  int box_atoms;
  float dt, invT;
  // plan
  const GemmUnit* gunits;
  const AttnUnit* aunits;  // cross-attention units (b, head, chunk)
  const CtaPlan* plans;
  const int* ctx_len;      // [B] valid context tokens
  // conditioning and small weights
  const float* mods;       // [S][L][3][3][768]
  const float* mod_final;  // [S][2][768]
  const float* rope_cos;   // [TMAX][48]
  const float* rope_sin;
  const float* bias[NUM_MATS];  // per layer: qkv [L][2304], so/cq/co/dn [L][768], gu = gate [L][3072] then up
  const float* b_up;            // [L][3072]
  const float* w_ain;   // [768][AD]
  const float* b_ain;   // [768]
  const float* w_aout;  // [AD][768] (bf16 values held in fp32)
  const float* b_aout;  // [AD]
  // cross-attention context (bound once), bf16, keys >= ctx_len zero: K [B][L][LKPAD][768] and V
  // transposed [B][L][768][LKPAD] (the K-major operand of O = P V)
  const __nv_bfloat16* kctx;
  const __nv_bfloat16* vctx;
  // state / scratch
  float* x_t;                 // [NT][AD]
  float* x;                   // [NPAD][768]
  float* part;                // [12][NPAD][768] K-split partials (self-out, cross-q, cross-out, down)
  __nv_bfloat16* xn;          // [NPAD][768]
  __nv_bfloat16* qkv;         // [NPAD][2304] self-attention q | k | v (+bias)
  __nv_bfloat16* sattn;       // [NPAD][768]
  __nv_bfloat16* cattn;       // [NPAD][768]
  __nv_bfloat16* hbuf;        // [NPAD][3072]
  __nv_bfloat16* opart;       // [B][8][MAX_CH][TMAX][96] per-chunk normalised cross-attention output
  float* oml;                 // [B][8][MAX_CH][TMAX][2] per-chunk (max log2, sum)
  // control
  unsigned int* bar;
  int* err;
  int wg;  // weight atoms per ring slot / TMA box
  // L2 prefetch distance of the weight stream, in layers (0 = off): the producer warp brings
  // this CTA's weight boxes of layer-step g + l2_ahead into L2 when it starts layer-step g.
  int l2_ahead;
  const uint8_t* wraw[kMaxMats];  // streamed weight matrices (bf16, or E4M3 codes), row-major [L * rows][K]
  int wrow_bytes[kMaxMats];        // bytes per weight row
  unsigned long long* stage_ns;
  int inject_barrier;
  unsigned int spin_limit;
  unsigned long long* trace;
  int trace_step, trace_layer;
};

}  // namespace ma2
}  // namespace fa
