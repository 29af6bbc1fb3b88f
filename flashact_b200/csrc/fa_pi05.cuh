// pi0.5 action-expert denoise megakernel: parameters and work plan shared by host and device.
//
// Reference semantics: src/pi05/mk6.cu:112-519 (loop body), src/pi05/hybrid_model.py:76-133
// (weight layout, modulations). Architecture constants are those of the Gemma-300M expert.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

#include "fa_engine_types.cuh"

namespace fa {
namespace pi05 {

constexpr int D = 1024;     // width
constexpr int H = 8;        // query heads (one shared KV head)
constexpr int HD = 256;     // head dim
constexpr int QD = H * HD;  // 2048
constexpr int F = 4096;     // GeGLU hidden
constexpr int QKV_ROWS = QD + 2 * HD;  // 2560
constexpr int MOD = 3 * D;  // scale|shift|gate
constexpr int TPAD = 64;    // action tokens padded per (observation, head) for attention tiles
constexpr int KCH = 128;    // prefix keys per attention chunk
constexpr int MAX_CH = 31;  // prefix chunks per observation (max_prefix <= 3968); index MAX_CH = action chunk

constexpr int kAttnWork = 160 * 1024;  // Q 64K | K/V 64K | P 32K

enum Mat : int { MAT_QKV = 0, MAT_O = 1, MAT_GU = 2, MAT_DN = 3 };
enum Map : int {
  MAP_W_QKV = 0, MAP_W_O, MAP_W_GU, MAP_W_DN,  // weights, box {64, 128}
  MAP_XN, MAP_ATTN, MAP_H,                     // activations, 3D box {64, NTILE, box_atoms}
  MAP_W_QKV_H, MAP_W_GU_H,                     // 64-row weight boxes of the half-row units
  MAP_Q, MAP_K, MAP_VT, MAP_SK, MAP_SVT,       // attention operands, 3D boxes of whole tiles
  NUM_MAPS
};
enum Stage : int {
  ST_NORM1 = 0, ST_QKV, ST_ATTN, ST_MERGE, ST_O, ST_NORM2, ST_GU, ST_DN, ST_FINAL, NUM_STAGES
};

struct Params {
  CUtensorMap maps[NUM_MAPS];
  // geometry
  int L, T, B, NT, NPAD, NTILE, TG, ngroups, nsteps, LPAD, AD;
  int split_o, split_dn;
  int tg[kMaxMats];  // token tiles per group (one accumulator) of each GEMM matrix
  int box_atoms;  // K atoms per activation TMA load (3D box)
  float dt;
  float invT;  // 1 / T
  // plan
  const GemmUnit* gunits;
  const AttnUnit* aunits;
  const CtaPlan* plans;
  const int* valid_len;  // [B]
  const int* nchunks;    // [B] prefix chunks (ceil(valid_len/128))
  // conditioning
  const float* mods;       // [S][L][2][3072]
  const float* mod_final;  // [S][3072]
  const float* rope_cos;   // [B][T][128]
  const float* rope_sin;
  const float* w_ain;   // [1024][AD]
  const float* b_ain;   // [1024]
  const float* w_aout;  // [AD][1024]
  const float* b_aout;  // [AD]
  // state / scratch
  float* x_t;      // [NT][AD]
  float* x;        // [NPAD][1024] residual stream
  float* part;     // [8][NPAD][1024] K-split partials
  __nv_bfloat16* xn;    // [NPAD][1024]
  __nv_bfloat16* attn;  // [NPAD][2048]
  __nv_bfloat16* hbuf;  // [NPAD][4096]
  __nv_bfloat16* q;     // [B][8][64][256]
  __nv_bfloat16* sk;    // [B][64][256] this layer's action-token keys (RoPE applied)
  __nv_bfloat16* svt;   // [B][256][64] this layer's action-token values, transposed
  __nv_bfloat16* opart;  // [B][4][MAX_CH+1][128][256] per-chunk normalised attention output (bf16)
  float* oml;    // [B][4][MAX_CH+1][128][2] per-chunk (max, sum)
  // control
  unsigned int* bar;             // grid-barrier counter, zeroed before each launch
  int* err;                      // 0 = ok; otherwise the first failure code
  int wg;  // weight atoms per ring slot / TMA box
  // L2 prefetch distance of the weight stream, in layers (0 = off): the producer warp brings
  // this CTA's weight boxes of layer-step g + l2_ahead into L2 when it starts layer-step g.
  int l2_ahead;
  const uint8_t* wraw[kMaxMats];  // streamed weight matrices (bf16, or E4M3 codes), row-major [L * rows][K]
  int wrow_bytes[kMaxMats];        // bytes per weight row
  // FP8 weight streaming: per packed weight row, its E4M3 scale, [L][rows] per matrix (QKV, O,
  // gate/up, down); unused by the bf16 kernel
  const float* wscale[4];
  int attn_whole;  // attention units cover all key chunks of (observation, head pair): two-pass softmax, no merge
  int f8_ahead;  // FP8 kernel: expand the next GEMM stage's first slots during the barrier before it
  unsigned long long* stage_ns;  // [NUM_STAGES] or null
  // host-side fault injection for tests: CTA 0 skips arriving at grid barrier number
  // `inject_barrier` (-1 = off); every grid-barrier spin gives up after `spin_limit` polls.
  int inject_barrier;
  unsigned int spin_limit;
  // optional trace of one (step, layer): per stage, per CTA, kTrStride clock64 stamps
  // (see TraceSlot); null = off.
  unsigned long long* trace;
  int trace_step, trace_layer;
};
}  // namespace pi05
}  // namespace fa
