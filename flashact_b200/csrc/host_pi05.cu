// Host side of the C ABI (include/flashact.h) for the pi0.5 engine: device buffers, on-device
// weight packing and conditioning, prefix-KV bind, work planning, TMA descriptors, launch.
#include "host_common.cuh"

using namespace fa;
using namespace fa::pi05;

thread_local std::string g_create_err;

namespace fa {
namespace pi05 {
__global__ void pi05_denoise_kernel(const __grid_constant__ Params p);
__global__ void pi05_denoise_kernel_f8(const __grid_constant__ Params p);
__global__ void pi05_denoise_kernel_tm(const __grid_constant__ Params p);
}
}  // namespace fa

// openpi create_sinusoidal_pos_embedding(t, 1024, min_period=4e-3, max_period=4.0):
// period_i = min * (max/min)^(i/511); emb = [sin(2 pi t / period) | cos(2 pi t / period)].
// Computed in double like the reference's float64 path, stored fp32. t_s = 1 - s/N.
__global__ void time_embed_kernel(float* emb, int S, int dim) {
  const int half = dim / 2;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < S * half; i += gridDim.x * blockDim.x) {
    const int s = i / half, j = i % half;
    const double frac = half > 1 ? (double)j / (double)(half - 1) : 0.0;
    const double period = 4e-3 * pow(4.0 / 4e-3, frac);
    const double t = 1.0 - (double)s / (double)S;
    const double arg = (2.0 * 3.14159265358979323846 / period) * (double)(float)t;
    emb[(size_t)s * dim + j] = (float)sin(arg);
    emb[(size_t)s * dim + half + j] = (float)cos(arg);
  }
}
// out[s][o] = act(b[o] + sum_i W[o][i] in[s][i]) for s < S; warp per output row; fp32 math.
// act: 0 none, 1 silu. out row s is at out + s * out_stride.
__global__ void linear_f32_kernel(const void* W, int wdt, const void* b, int bdt, const float* in, int S, int IN,
                                  int OUT, float* out, size_t out_stride, int act) {
  extern __shared__ float xs[];  // [S][IN]
  for (int i = threadIdx.x; i < S * IN; i += blockDim.x) xs[i] = in[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (int o = blockIdx.x * warps + (threadIdx.x >> 5); o < OUT; o += gridDim.x * warps) {
    float acc[16];
    for (int s0 = 0; s0 < S; s0 += 16) {
      const int ns = min(16, S - s0);
#pragma unroll
      for (int s = 0; s < 16; ++s) acc[s] = 0.f;
      for (int i = lane; i < IN; i += 32) {
        const float w = load_as_float(W, (size_t)o * IN + i, wdt);
#pragma unroll
        for (int s = 0; s < 16; ++s)
          if (s < ns) acc[s] = fmaf(w, xs[(s0 + s) * IN + i], acc[s]);
      }
#pragma unroll
      for (int s = 0; s < 16; ++s) {
        float v = acc[s];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0 && s < ns) {
          v += load_as_float(b, o, bdt);
          if (act == 1) v = v / (1.f + expf(-v));
          out[(size_t)(s0 + s) * out_stride + o] = v;
        }
      }
    }
  }
}
// Prefix KV bind: K -> kcache[b][l][LPAD][256] (split-half RoPE order), V -> vtcache[b][l][256][LPAD]
// (transposed), rows >= valid_len zero. Interleaved sources (FlashRT) have rotary pairs at
// (2d, 2d+1): d -> d, d+1 -> d+128 (src/pi05/mk6.cu:258-277 does the same de-interleave).
__global__ void bind_k_kernel(const bf16* k, int src_rows, const int* valid, const int* rowmap, int L, int LPAD,
                              int interleaved, bf16* kc) {
  const int b = blockIdx.z, l = blockIdx.y;
  const int vl = valid[b];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < LPAD * HD; i += gridDim.x * blockDim.x) {
    const int r = i / HD, d = i % HD;
    bf16 v = __float2bfloat16(0.f);
    if (r < vl) {
      int sd = d;
      if (interleaved) sd = d < 128 ? 2 * d : 2 * (d - 128) + 1;
      const int sr = rowmap ? rowmap[(size_t)b * src_rows + r] : r;  // kept row of a masked bind
      v = k[(((size_t)b * L + l) * src_rows + sr) * HD + sd];
    }
    kc[(((size_t)b * L + l) * LPAD + r) * HD + d] = v;
  }
}
__global__ void bind_vt_kernel(const bf16* v, int src_rows, const int* valid, const int* rowmap, int L, int LPAD,
                               bf16* vt) {
  __shared__ bf16 tile[32][33];
  const int b = blockIdx.z / L, l = blockIdx.z % L;
  const int vl = valid[b];
  const int r0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, d = d0 + threadIdx.x;
    const int sr = rowmap && r < vl ? rowmap[(size_t)b * src_rows + r] : r;
    tile[i][threadIdx.x] = r < vl ? v[(((size_t)b * L + l) * src_rows + sr) * HD + d] : __float2bfloat16(0.f);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int d = d0 + i, r = r0 + threadIdx.x;
    vt[(((size_t)b * L + l) * HD + d) * LPAD + r] = tile[threadIdx.x][i];
  }
}
// RoPE tables for the action tokens: pos = valid_len[b] + t, inv_freq_i = 10000^(-2i/256)
// (src/pi05/pack_weights.py:54-58), angle = fp32(pos) * fp32(inv_freq) as in the fp32 reference.
__global__ void rope_kernel(const int* valid, int B, int T, float* cs, float* sn) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < B * T * 128; i += gridDim.x * blockDim.x) {
    const int j = i % 128, t = (i / 128) % T, b = i / (128 * T);
    const float inv = (float)(1.0 / pow(10000.0, (double)(2 * j) / 256.0));
    const float ang = (float)(valid[b] + t) * inv;
    cs[i] = (float)cos((double)ang);
    sn[i] = (float)sin((double)ang);
  }
}

// ------------------------------------------------------------------ create / destroy

extern "C" fa_status fa_create(fa_model_kind kind, const fa_config* cfg, int device, fa_handle** out) {
  if (!cfg || !out) return fail(nullptr, FA_ERR_INVALID, "null argument");
  *out = nullptr;
  if (kind != FA_MODEL_PI05 && kind != FA_MODEL_MOLMOACT2)
    return fail(nullptr, FA_ERR_UNSUPPORTED, "model kind %d not built into this library", (int)kind);
  const fa_config& c = *cfg;
  if (kind == FA_MODEL_MOLMOACT2) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
      cudaGetLastError();
      return fail(nullptr, FA_ERR_INVALID, "device %d not available", device);
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return fail(nullptr, FA_ERR_CUDA, "cudaGetDeviceProperties failed");
    if (prop.major != 10 || prop.minor != 0)
      return fail(nullptr, FA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a (B200)", device, prop.major, prop.minor);
    fa_handle* h = new fa_handle();
    h->kind = kind;
    h->cfg = c;
    h->device = device;
    h->num_sms = prop.multiProcessorCount;
    h->params.inject_barrier = -1;  // fault injection off
    h->params.spin_limit = 1u << 24;
    const fa_status st = ma2_create(c, device, h);
    if (st != FA_OK) {
      g_create_err = h->err;
      fa_destroy(h);
      return st;
    }
    *out = h;
    return FA_OK;
  }
  if (c.width != D || c.num_heads != H || c.num_kv_heads != 1 || c.head_dim != HD || c.mlp_dim != F)
    return fail(nullptr, FA_ERR_INVALID, "pi0.5 expert geometry must be width 1024, 8 heads, 1 kv head, head_dim 256, mlp 4096");
  if (c.num_layers < 1 || c.num_layers > 64 || c.horizon < 1 || c.horizon > TPAD || c.action_dim < 1 || c.action_dim > 32 ||
      c.max_prefix < 0 || c.max_prefix > MAX_CH * KCH || c.max_batch < 1 || c.max_batch > 1024 || c.num_steps < 1 ||
      c.num_steps > 50)
    return fail(nullptr, FA_ERR_INVALID,
                "config out of range (layers 1..64, horizon 1..64, action_dim 1..32, max_prefix 0..3968, batch 1..1024, steps 1..50)");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    return fail(nullptr, FA_ERR_INVALID, "device %d not available", device);
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return fail(nullptr, FA_ERR_CUDA, "cudaGetDeviceProperties failed");
  if (prop.major != 10 || prop.minor != 0)
    return fail(nullptr, FA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a (B200)", device, prop.major, prop.minor);
  if (!prop.cooperativeLaunch) return fail(nullptr, FA_ERR_UNSUPPORTED, "device lacks cooperative launch");

  fa_handle* h = new fa_handle();
  h->kind = kind;
  h->cfg = c;
  h->device = device;
  h->num_sms = prop.multiProcessorCount;
  // K-split factors (tuning knobs): powers of two, so that every unit covers a multiple of 4 atoms
  auto pow2 = [](int v) { int r = 1; while (r * 2 <= v) r *= 2; return r; };
  if (const char* e = getenv("FA_SPLIT_O")) h->split_o = pow2(std::max(1, std::min(8, atoi(e))));
  if (const char* e = getenv("FA_SPLIT_DN")) h->split_dn = pow2(std::max(1, std::min(8, atoi(e))));
  if (const char* e = getenv("FA_RING_MAX")) h->ring_max = std::max(2, atoi(e));
  if (const char* e = getenv("FA_HALF_UNITS")) h->half_units = atoi(e) != 0;
  if (const char* e = getenv("FA_BMAX_KB")) h->bmax_bytes = std::max(8, std::min(128, atoi(e))) * 1024;
  if (const char* e = getenv("FA_ATTN_PENALTY")) h->attn_penalty = std::max(0, atoi(e));
  auto bad = [&](fa_status st) { g_create_err = h->err; fa_destroy(h); return st; };
  if (cudaSetDevice(device) != cudaSuccess) return bad(fail(h, FA_ERR_CUDA, "cudaSetDevice(%d) failed", device));

  const int L = c.num_layers, T = c.horizon, S = c.num_steps, MB = c.max_batch;
  const int NPADm = round_up(MB * T, 128);
  const int LPADm = std::max(KCH, round_up(c.max_prefix, KCH));
  fa_status st = FA_OK;
#define ALLOC(ptr, n) if ((st = dalloc(h, &h->ptr, (size_t)(n))) != FA_OK) return bad(st)
  ALLOC(w_qkv, (size_t)L * QKV_ROWS * D);
  ALLOC(w_o, (size_t)L * D * QD);
  ALLOC(w_gu, (size_t)L * 2 * F * D);
  ALLOC(w_dn, (size_t)L * D * F);
  ALLOC(mods, (size_t)S * L * 2 * MOD);
  ALLOC(mod_final, (size_t)S * MOD);
  ALLOC(w_ain, (size_t)D * c.action_dim);
  ALLOC(b_ain, D);
  ALLOC(w_aout, (size_t)c.action_dim * D);
  ALLOC(b_aout, c.action_dim);
  ALLOC(x_t, (size_t)NPADm * c.action_dim);
  ALLOC(x, (size_t)NPADm * D);
  ALLOC(part, (size_t)8 * NPADm * D);
  ALLOC(xn, (size_t)NPADm * D);
  ALLOC(attn, (size_t)NPADm * QD);
  ALLOC(hbuf, (size_t)NPADm * F);
  ALLOC(q, (size_t)MB * H * TPAD * HD);
  ALLOC(sk, (size_t)MB * TPAD * HD);
  ALLOC(svt, (size_t)MB * HD * TPAD);
  ALLOC(opart, (size_t)MB * 4 * (MAX_CH + 1) * 128 * HD);
  ALLOC(oml, (size_t)MB * 4 * (MAX_CH + 1) * 128 * 2);
  ALLOC(kcache, (size_t)MB * L * LPADm * HD);
  ALLOC(vtcache, (size_t)MB * L * HD * LPADm);
  ALLOC(rope_cos, (size_t)MB * T * 128);
  ALLOC(rope_sin, (size_t)MB * T * 128);
  ALLOC(d_valid, MB);
  ALLOC(d_nchunks, MB);
  ALLOC(ctrl, kCtrlWords);
  ALLOC(stage_ns, kMaxStages);
  ALLOC(d_plans, h->num_sms);
#undef ALLOC
  const void* kernels[3] = {(const void*)fa::pi05::pi05_denoise_kernel, (const void*)fa::pi05::pi05_denoise_kernel_f8,
                            (const void*)fa::pi05::pi05_denoise_kernel_tm};
  const int threads[3] = {kThreads, kThreads, kThreads};
  for (int i = 0; i < 3; ++i) {
    if (cudaFuncSetAttribute(kernels[i], cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemDyn) != cudaSuccess)
      return bad(fail(h, FA_ERR_CUDA, "cannot reserve %d bytes of shared memory", kSmemDyn));
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernels[i], threads[i], kSmemDyn) != cudaSuccess || occ < 1)
      return bad(fail(h, FA_ERR_UNSUPPORTED, "megakernel %d does not fit on an SM (occupancy %d)", i, occ));
  }
  *out = h;
  return FA_OK;
}

extern "C" void fa_destroy(fa_handle* h) {
  if (!h) return;
  cudaSetDevice(h->device);
  ma2_destroy(h);
  for (void* p : h->allocs) cudaFree(p);
  delete h;
}

extern "C" const char* fa_last_error(fa_handle* h) { return h ? h->err.c_str() : g_create_err.c_str(); }
extern "C" int fa_last_launch_count(fa_handle* h) { return h ? h->last_launches : 0; }

// ------------------------------------------------------------------ weights
static fa_status run_linear(fa_handle* h, const void* W, fa_dtype wdt, const void* b, fa_dtype bdt, const float* in, int S,
                            int IN, int OUT, float* out, size_t out_stride, int act) {
  const size_t smem = (size_t)S * IN * sizeof(float);
  if (smem > 48 * 1024) FA_CUDA(h, cudaFuncSetAttribute(linear_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  linear_f32_kernel<<<h->num_sms * 2, 256, smem>>>(W, wdt, b, bdt, in, S, IN, OUT, out, out_stride, act);
  FA_CUDA(h, cudaGetLastError());
  return FA_OK;
}

static fa_status load_weights_impl(fa_handle* h, const fa_pi05_weights* w, fa_wfmt fmt, const fa_pi05_qscales* q);
static fa_status build_plan(fa_handle* h);
static fa_status build_params(fa_handle* h);

// The plan and tensor maps depend on the weight format (FP8 streaming or bf16): a bound batch
// is re-planned when weights are (re)loaded after the bind.
static fa_status weights_loaded(fa_handle* h) {
  h->weights_ready = true;
  if (!h->kv_ready) return FA_OK;
  fa_status st = build_plan(h);
  return st != FA_OK ? st : build_params(h);
}

extern "C" fa_status fa_pi05_load_weights(fa_handle* h, const fa_pi05_weights* w, fa_wfmt fmt) {
  if (!h || !w) return fail(h, FA_ERR_INVALID, "null argument");
  if (fmt != FA_WFMT_BF16)
    return fail(h, FA_ERR_INVALID, "quantised weights go through fa_pi05_load_weights_q (they need scales)");
  return load_weights_impl(h, w, fmt, nullptr);
}

extern "C" fa_status fa_pi05_load_weights_q(fa_handle* h, const fa_pi05_weights* w, fa_wfmt fmt,
                                            const fa_pi05_qscales* q) {
  if (!h || !w || !q) return fail(h, FA_ERR_INVALID, "null argument");
  if (fmt != FA_WFMT_FP8 && fmt != FA_WFMT_NVFP4) return fail(h, FA_ERR_INVALID, "unknown quantised format %d", (int)fmt);
  return load_weights_impl(h, w, fmt, q);
}

static fa_status load_weights_impl(fa_handle* h, const fa_pi05_weights* w, fa_wfmt fmt, const fa_pi05_qscales* q) {
  if (h->kind != FA_MODEL_PI05) return fail(h, FA_ERR_INVALID, "not a pi0.5 handle");
  FA_CUDA(h, cudaSetDevice(h->device));
  const int L = h->cfg.num_layers, AD = h->cfg.action_dim, S = h->cfg.num_steps;
  std::vector<void*> tmp;
  struct Cleanup {
    std::vector<void*>& t;
    ~Cleanup() { for (void* p : t) cudaFree(p); }
  } cleanup{tmp};
  fa_status st;
  const void *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr, *wg = nullptr, *wu = nullptr, *wd = nullptr,
             *lniw = nullptr, *lnib = nullptr, *lnpw = nullptr, *lnpb = nullptr, *nw = nullptr, *nb = nullptr,
             *tiw = nullptr, *tib = nullptr, *tow = nullptr, *tob = nullptr, *aiw = nullptr, *aib = nullptr,
             *aow = nullptr, *aob = nullptr;
  // The conditioning weights (time MLP, adaRMS denses) are optional as a group: without them the
  // caller supplies the modulations with fa_set_modulation, as the reference's launch() takes them.
  const fa_tensor* cond_w[10] = {&w->ln_in_w, &w->ln_in_b, &w->ln_post_w, &w->ln_post_b, &w->norm_w,
                               &w->norm_b,  &w->time_in_w, &w->time_in_b, &w->time_out_w, &w->time_out_b};
  int ncond = 0;
  for (const fa_tensor* t : cond_w) ncond += t->ptr != nullptr;
  if (ncond != 0 && ncond != 10)
    return fail(h, FA_ERR_INVALID, "conditioning weights must be all given or all null (%d of 10 given)", ncond);
  const bool with_cond = ncond == 10;
#define STAGE(var, field, count) \
  if ((st = stage_tensor(h, w->field, (size_t)(count), #field, &var, tmp)) != FA_OK) return st
  // GEMM weights: plain tensors, or codes + scales of a quantised format
  const int qmode = fmt == FA_WFMT_FP8 ? 1 : fmt == FA_WFMT_NVFP4 ? 2 : 0;
  const void* qs[7] = {nullptr};   // row (FP8) or block (NVFP4) scales, device
  const float* qt[7] = {nullptr};  // NVFP4 per-layer tensor scales, device
  {
    const fa_tensor* wt[7] = {&w->wq, &w->wk, &w->wv, &w->wo, &w->w_gate, &w->w_up, &w->w_down};
    const void** dst[7] = {&wq, &wk, &wv, &wo, &wg, &wu, &wd};
    const int rows[7] = {QD, HD, HD, D, F, F, D}, cols[7] = {D, D, D, QD, D, D, F};
    const char* names[7] = {"wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"};
    const fa_qscale* sc[7] = {q ? &q->wq : nullptr, q ? &q->wk : nullptr, q ? &q->wv : nullptr, q ? &q->wo : nullptr,
                              q ? &q->w_gate : nullptr, q ? &q->w_up : nullptr, q ? &q->w_down : nullptr};
    for (int i = 0; i < 7; ++i) {
      const size_t n = (size_t)L * rows[i] * cols[i];
      if (qmode == 0) {
        if ((st = stage_tensor(h, *wt[i], n, names[i], dst[i], tmp)) != FA_OK) return st;
        continue;
      }
      if ((st = stage_bytes(h, wt[i]->ptr, qmode == 1 ? n : n / 2, names[i], dst[i], tmp)) != FA_OK) return st;
      const size_t sbytes = qmode == 1 ? (size_t)L * rows[i] * 4 : n / 16;
      if ((st = stage_bytes(h, sc[i]->scale, sbytes, names[i], &qs[i], tmp)) != FA_OK) return st;
      if (qmode == 2) {
        const void* t = nullptr;
        if ((st = stage_bytes(h, sc[i]->tensor, (size_t)L * 4, names[i], &t, tmp)) != FA_OK) return st;
        qt[i] = reinterpret_cast<const float*>(t);
      }
    }
  }
  if (with_cond) {
    STAGE(lniw, ln_in_w, (size_t)L * MOD * D);
    STAGE(lnib, ln_in_b, (size_t)L * MOD);
    STAGE(lnpw, ln_post_w, (size_t)L * MOD * D);
    STAGE(lnpb, ln_post_b, (size_t)L * MOD);
    STAGE(nw, norm_w, (size_t)MOD * D);
    STAGE(nb, norm_b, MOD);
    STAGE(tiw, time_in_w, (size_t)D * D);
    STAGE(tib, time_in_b, D);
    STAGE(tow, time_out_w, (size_t)D * D);
    STAGE(tob, time_out_b, D);
  }
  STAGE(aiw, ain_w, (size_t)D * AD);
  STAGE(aib, ain_b, D);
  STAGE(aow, aout_w, (size_t)AD * D);
  STAGE(aob, aout_b, AD);
#undef STAGE

  // QKV rows: Q head h / K in 128-row tiles where row 32*q + lane holds rotary pair
  // p = 64*pb + 16*q + (lane & 15), dim p + 128*(lane >> 4); V rows in natural order.
  std::vector<int2> m1(QKV_ROWS);
  for (int mt = 0; mt < 20; ++mt)
    for (int r = 0; r < 128; ++r) {
      const int qd = r >> 5, lane = r & 31;
      if (mt < 18) {
        const int pb = mt < 16 ? (mt & 1) : mt - 16;
        const int dim = 64 * pb + 16 * qd + (lane & 15) + 128 * (lane >> 4);
        m1[mt * 128 + r] = mt < 16 ? make_int2(0, (mt >> 1) * HD + dim) : make_int2(1, dim);
      } else {
        m1[mt * 128 + r] = make_int2(2, (mt - 18) * 128 + r);
      }
    }
  PackSrc s1 = {{wq, wk, wv}, {w->wq.dtype, w->wk.dtype, w->wv.dtype}, {QD, HD, HD}, qmode, {qs[0], qs[1], qs[2]},
                {qt[0], qt[1], qt[2]}};
  // FP8 codes are streamed as they are (the FP8 kernel; FA_FP8_STREAM=0 dequantises to bf16
  // instead); the other formats are dequantised once into the bf16 layout.
  const char* fs = getenv("FA_FP8_STREAM");
  h->fp8_stream = qmode == 1 && !(fs && atoi(fs) == 0);
  if (h->fp8_stream) {
    const void* codes[7] = {wq, wk, wv, wo, wg, wu, wd};
    for (const void* cp : codes)
      if (reinterpret_cast<uintptr_t>(cp) % 16) return fail(h, FA_ERR_INVALID, "FP8 codes must be 16-byte aligned");
    const size_t rows4[4] = {(size_t)QKV_ROWS, (size_t)D, (size_t)2 * F, (size_t)D}, k4[4] = {D, QD, D, F};
    for (int m = 0; m < 4; ++m) {
      if (!h->w8[m] && (st = dalloc(h, &h->w8[m], (size_t)L * rows4[m] * k4[m])) != FA_OK) return st;
      if (!h->ws8[m] && (st = dalloc(h, &h->ws8[m], (size_t)L * rows4[m])) != FA_OK) return st;
    }
  }
  if (h->fp8_stream) {
    if ((st = pack_codes(h, m1, s1, h->w8[0], h->ws8[0], D, tmp)) != FA_OK) return st;
  } else if ((st = pack_matrix(h, m1, s1, h->w_qkv, D, tmp)) != FA_OK) {
    return st;
  }
  std::vector<int2> mo(D);
  for (int r = 0; r < D; ++r) mo[r] = make_int2(0, r);
  PackSrc so = {{wo, wo, wo}, {w->wo.dtype, w->wo.dtype, w->wo.dtype}, {D, D, D}, qmode, {qs[3], qs[3], qs[3]},
                {qt[3], qt[3], qt[3]}};
  if (h->fp8_stream) {
    if ((st = pack_codes(h, mo, so, h->w8[1], h->ws8[1], QD, tmp)) != FA_OK) return st;
  } else if ((st = pack_matrix(h, mo, so, h->w_o, QD, tmp)) != FA_OK) {
    return st;
  }
  // gate/up rows: tile mt, row 32*q + lane -> feature 64*mt + 16*q + (lane & 15); lanes < 16 gate.
  std::vector<int2> m2(2 * F);
  for (int mt = 0; mt < 64; ++mt)
    for (int r = 0; r < 128; ++r) {
      const int qd = r >> 5, lane = r & 31;
      m2[mt * 128 + r] = make_int2(lane < 16 ? 0 : 1, 64 * mt + 16 * qd + (lane & 15));
    }
  PackSrc s2 = {{wg, wu, wu}, {w->w_gate.dtype, w->w_up.dtype, w->w_up.dtype}, {F, F, F}, qmode, {qs[4], qs[5], qs[5]},
                {qt[4], qt[5], qt[5]}};
  if (h->fp8_stream) {
    if ((st = pack_codes(h, m2, s2, h->w8[2], h->ws8[2], D, tmp)) != FA_OK) return st;
  } else if ((st = pack_matrix(h, m2, s2, h->w_gu, D, tmp)) != FA_OK) {
    return st;
  }
  PackSrc s3 = {{wd, wd, wd}, {w->w_down.dtype, w->w_down.dtype, w->w_down.dtype}, {D, D, D}, qmode,
                {qs[6], qs[6], qs[6]}, {qt[6], qt[6], qt[6]}};
  if (h->fp8_stream) {
    if ((st = pack_codes(h, mo, s3, h->w8[3], h->ws8[3], F, tmp)) != FA_OK) return st;
  } else if ((st = pack_matrix(h, mo, s3, h->w_dn, F, tmp)) != FA_OK) {
    return st;
  }

  to_f32_kernel<<<64, 256>>>(aiw, w->ain_w.dtype, h->w_ain, (size_t)D * AD);
  to_f32_kernel<<<4, 256>>>(aib, w->ain_b.dtype, h->b_ain, D);
  to_f32_kernel<<<64, 256>>>(aow, w->aout_w.dtype, h->w_aout, (size_t)AD * D);
  to_f32_kernel<<<1, 64>>>(aob, w->aout_b.dtype, h->b_aout, AD);
  FA_CUDA(h, cudaGetLastError());

  if (!with_cond) {  // modulations come from fa_set_modulation
    FA_CUDA(h, cudaDeviceSynchronize());
    return weights_loaded(h);
  }
  // Conditioning for the fixed schedule t_s = 1 - s/N (src/pi05/hybrid_model.py:111-128):
  // cond = silu(W_out silu(W_in emb + b_in) + b_out); mods = Dense_{in,post}(cond); final = Dense_norm(cond).
  float *emb = nullptr, *h1 = nullptr, *cond = nullptr;
  FA_CUDA(h, cudaMalloc(&emb, (size_t)S * D * 4));
  tmp.push_back(emb);
  FA_CUDA(h, cudaMalloc(&h1, (size_t)S * D * 4));
  tmp.push_back(h1);
  FA_CUDA(h, cudaMalloc(&cond, (size_t)S * D * 4));
  tmp.push_back(cond);
  time_embed_kernel<<<8, 256>>>(emb, S, D);
  FA_CUDA(h, cudaGetLastError());
  if ((st = run_linear(h, tiw, w->time_in_w.dtype, tib, w->time_in_b.dtype, emb, S, D, D, h1, D, 1)) != FA_OK) return st;
  if ((st = run_linear(h, tow, w->time_out_w.dtype, tob, w->time_out_b.dtype, h1, S, D, D, cond, D, 1)) != FA_OK) return st;
  const size_t sstride = (size_t)L * 2 * MOD;
  for (int l = 0; l < L; ++l) {
    const size_t wo_ = (size_t)l * MOD * D * dtype_size(w->ln_in_w.dtype);
    const size_t bo_ = (size_t)l * MOD * dtype_size(w->ln_in_b.dtype);
    if ((st = run_linear(h, (const char*)lniw + wo_, w->ln_in_w.dtype, (const char*)lnib + bo_, w->ln_in_b.dtype, cond, S, D,
                         MOD, h->mods + (size_t)l * 2 * MOD, sstride, 0)) != FA_OK)
      return st;
    const size_t wp_ = (size_t)l * MOD * D * dtype_size(w->ln_post_w.dtype);
    const size_t bp_ = (size_t)l * MOD * dtype_size(w->ln_post_b.dtype);
    if ((st = run_linear(h, (const char*)lnpw + wp_, w->ln_post_w.dtype, (const char*)lnpb + bp_, w->ln_post_b.dtype, cond, S,
                         D, MOD, h->mods + (size_t)l * 2 * MOD + MOD, sstride, 0)) != FA_OK)
      return st;
  }
  if ((st = run_linear(h, nw, w->norm_w.dtype, nb, w->norm_b.dtype, cond, S, D, MOD, h->mod_final, MOD, 0)) != FA_OK) return st;
  FA_CUDA(h, cudaDeviceSynchronize());
  return weights_loaded(h);
}

extern "C" fa_status fa_set_modulation(fa_handle* h, const float* mods, const float* mod_final) {
  if (!h || !mods || !mod_final) return fail(h, FA_ERR_INVALID, "null argument");
  if (h->kind == FA_MODEL_MOLMOACT2) return ma2_set_modulation(h, mods, mod_final);
  FA_CUDA(h, cudaSetDevice(h->device));
  const size_t n = (size_t)h->cfg.num_steps * h->cfg.num_layers * 2 * MOD;
  FA_CUDA(h, cudaMemcpy(h->mods, mods, n * 4, cudaMemcpyDefault));
  FA_CUDA(h, cudaMemcpy(h->mod_final, mod_final, (size_t)h->cfg.num_steps * MOD * 4, cudaMemcpyDefault));
  return FA_OK;
}

// ------------------------------------------------------------------ work plan
// GEMM units per layer: QKV 20 x 128-row tiles (full K), O 8 tiles x split_o K-slices,
// gate/up 64 tiles (full K), down 8 tiles x split_dn K-slices. Attention units: per
// observation, 4 head pairs x (prefix chunks + 1 suffix chunk). Attention units go to the first
// CTAs in contiguous runs (same head pair -> Q reuse); each GEMM stage is then spread so that
// no CTA holds two units of one stage before all CTAs hold one, ties broken by total bytes.
// K atoms per activation TMA load (32 KB boxes).
// Never more than divides every unit's K range (O and down are K-split).
static int act_box_atoms(const fa_handle* h) {
  int ba = h->NTILE == 64 ? 4 : 2;
  while (ba > 1 && ((QD / 64 / h->split_o_eff) % ba != 0 || (F / 64 / h->split_dn_eff) % ba != 0)) ba >>= 1;
  return ba;
}

// 64-row units for QKV and gate/up while the bound batch is one 64-token tile.
static bool use_half_units(const fa_handle* h) { return h->half_units && h->NTILE == 64 && h->ngroups == 1; }

static fa_status build_plan(fa_handle* h) {
  const int nblk = h->num_sms;
  // token tiles per group = per TMEM accumulator: 256 columns, or 128 with FP8 streaming (the
  // upper half of TMEM holds the expanded weight slots)
  h->TG = (h->fp8_stream ? kAccColsF8 : 256) / h->NTILE;
  if (const char* e = getenv("FA_TG_MAX")) h->TG = std::max(1, std::min(h->TG, atoi(e)));  // tuning knob
  h->ngroups = (h->NPAD / h->NTILE + h->TG - 1) / h->TG;
  // QKV at 128-token tiles: one tile per unit. Its units then each read a quarter or half of the
  // activation of a 2-tile group (the activation, not the 5.2 MB of weights, dominates what a QKV
  // CTA loads once the batch spans several tiles); measured at bs=8: QKV 7.4 -> 5.3 ms per chunk.
  const int tiles = h->NPAD / h->NTILE;
  for (int m = 0; m < 4; ++m) h->tgm[m] = h->TG;
  if (h->NTILE == 128) {
    const char* e = getenv("FA_QKV_TG");
    h->tgm[MAT_QKV] = std::max(1, std::min(h->TG, e ? atoi(e) : 1));
  }
  auto ngr = [&](int m) { return (tiles + h->tgm[m] - 1) / h->tgm[m]; };
  auto ntiles_of = [&](int m, int g) { return std::min(h->tgm[m], tiles - g * h->tgm[m]); };
  // Attention units: per (observation, head pair, key chunk) with a merge stage (split-KV: the
  // latency choice at a few observations), or per (observation, head pair) over all its chunks
  // (two-pass softmax, no partials: the throughput choice once the units alone fill the GPU).
  {
    const char* e = getenv("FA_ATTN_WHOLE");
    h->attn_whole = e ? atoi(e) != 0 : 8 * h->B >= nblk;  // measured: 32 obs 53.9 -> 46.9 ms, 16 obs 33.1 -> 34.0
  }
  std::vector<AttnUnit> au;
  for (int b = 0; b < h->B; ++b) {
    const int npc = (h->valid_len[b] + KCH - 1) / KCH;
    for (int hp = 0; hp < 4; ++hp) {
      if (h->attn_whole) {
        au.push_back({(uint16_t)b, (uint16_t)hp, kWholeChunk, 0});
        continue;
      }
      for (int c = 0; c < npc; ++c) au.push_back({(uint16_t)b, (uint16_t)hp, (uint16_t)c, 0});
      au.push_back({(uint16_t)b, (uint16_t)hp, 0, 1});
    }
  }
  std::vector<CtaPlan> plans(nblk);
  std::vector<long> load(nblk, 0);
  const int na = (int)au.size();
  const int acta = std::min(na, nblk);
  for (int i = 0; i < nblk; ++i) {
    const int lo = i < acta ? (int)((long)na * i / acta) : 0, hi = i < acta ? (int)((long)na * (i + 1) / acta) : 0;
    plans[i].a_off = lo;
    plans[i].a_cnt = hi - lo;
    load[i] = (long)plans[i].a_cnt * h->attn_penalty;
  }
  // K-splits of O and down: the configured factor, halved while the stage would hold more than
  // two units per CTA (large batches fill the GPU through their token groups instead).
  auto eff_split = [&](int mtiles, int split) {
    while (split > 1 && mtiles * split * h->ngroups > 2 * nblk) split >>= 1;
    return split;
  };
  h->split_o_eff = eff_split(8, h->split_o);
  h->split_dn_eff = eff_split(8, h->split_dn);
  struct Spec { int mtiles, katoms, split; };
  const Spec spec[4] = {{20, D / 64, 1}, {8, QD / 64, h->split_o_eff}, {64, D / 64, 1}, {8, F / 64, h->split_dn_eff}};
  // Weight atoms per ring slot: 64 KB boxes when one token tile is in flight, 32 KB otherwise
  // (keeps an attention CTA's activation batch, which must hold whole slots, inside 64 KB); never
  // more than divides every unit's K range.
  // Token-major GEMMs (pi05_denoise_kernel_tm) while the batch is one tile of <= 64 tokens with
  // bf16 weights and every unit's K range is whole 4-atom chunks (FA_TM=0 keeps the weight-major
  // kernel). Their CTAs stage a unit's activation K-chunks (32 KB each, four on CTAs without
  // attention units) beside the weight ring, which then holds 32 KB boxes.
  {
    const char* e = getenv("FA_TM");
    bool tm = !(e && atoi(e) == 0) && !h->fp8_stream && use_half_units(h) && act_box_atoms(h) == kTmChunkAtoms;
    for (int m = 0; m < 4; ++m) tm = tm && (spec[m].katoms / spec[m].split) % kTmChunkAtoms == 0;
    h->tm = tm;
  }
  h->wg = h->tm ? 2 : h->NTILE == 64 ? kMaxWG : 2;  // token-major: 32 KB boxes (its MMA issue assumes 2 atoms)
  if (const char* e = getenv("FA_WG"); e && !h->tm) h->wg = std::max(1, std::min(h->wg, atoi(e)));
  // FP8 streaming: 2 atoms per slot (one 128 x 128-byte E4M3 box, expanded to 32 KB of bf16)
  if (h->fp8_stream) h->wg = 2;
  for (int m = 0; m < 4; ++m)
    while ((spec[m].katoms / spec[m].split) % h->wg != 0) h->wg >>= 1;
  if (h->tm && h->wg != 2) return fail(h, FA_ERR_INVALID, "plan error: token-major GEMMs need 2-atom weight boxes");
  // QKV also runs as 64-row units while its 128-row units would leave most SMs idle (20 tiles per
  // token group: at a few observations per GPU the stage is otherwise carried by 20 x groups
  // CTAs), provided every CTA that can receive one has room for its activation batch: an
  // attention CTA's area is 64 KB, and the planner fills the CTAs without attention units first.
  const int ntg_max = std::min(h->tgm[MAT_QKV], tiles);
  const bool half_fits_attn = h->NTILE * 128 * ntg_max * std::max(act_box_atoms(h), 2 * h->wg) <= 64 * 1024;
  const bool qkv_half = use_half_units(h) ||
                        (h->half_units && 40 * ngr(MAT_QKV) <= (half_fits_attn ? nblk : nblk - acta));
  std::vector<std::vector<GemmUnit>> per(nblk * 4);
  const int order[4] = {MAT_QKV, MAT_GU, MAT_DN, MAT_O};
  for (int oi = 0; oi < 4; ++oi) {
    const int m = order[oi];
    const Spec& s = spec[m];
    const int per_split = s.katoms / s.split;
    // QKV and gate/up at one 64-token tile: 64-row units (each SM streams half a tile, which its
    // weight ring holds whole; RoPE / GeGLU partners stay in one unit)
    const int halves = ((m == MAT_QKV && qkv_half) || (m == MAT_GU && use_half_units(h))) ? 2 : 1;
    std::vector<int> cnt(nblk, 0);
    for (int g = 0; g < ngr(m); ++g)
      for (int mt = 0; mt < s.mtiles; ++mt)
        for (int hf = 0; hf < halves; ++hf)
          for (int sp = 0; sp < s.split; ++sp) {
            int best = 0;
            for (int i = 1; i < nblk; ++i)
              if (cnt[i] < cnt[best] || (cnt[i] == cnt[best] && load[i] < load[best])) best = i;
            per[best * 4 + m].push_back({(uint16_t)mt, (uint16_t)(sp * per_split), (uint16_t)per_split, (uint16_t)sp,
                                         (uint16_t)g, (uint16_t)(halves == 2 ? hf + 1 : 0)});
            cnt[best]++;
            load[best] += per_split * ntiles_of(m, g) / halves;
          }
  }
  std::vector<GemmUnit> gu;
  const int tile = h->NTILE * 128;
  for (int i = 0; i < nblk; ++i) {
    // Activation area: the largest (unit, token group) K-range of this CTA, whole if it fits.
    int bb = tile, ng = 0, ntg = 1;  // ntg: most token tiles of a unit of this CTA
    for (int m = 0; m < 4; ++m) {
      ng += (int)per[i * 4 + m].size();
      for (const GemmUnit& x : per[i * 4 + m]) {
        bb = std::max(bb, (int)x.natoms * ntiles_of(m, x.grp) * tile);
        ntg = std::max(ntg, ntiles_of(m, x.grp));
      }
    }
    if (ng > kMaxGU || plans[i].a_cnt > kMaxAU)
      return fail(h, FA_ERR_INVALID, "batch too large for the per-CTA work lists (%d GEMM, %d attention units)", ng,
                  plans[i].a_cnt);
    // Capped so that the weight ring stays deep (larger K ranges load in several batches).
    bb = std::min(bb, std::min(std::min(kMaxBBytes, h->bmax_bytes), kMaxBAtoms * tile));
    bb = std::max(bb, tile * ntg * std::max(act_box_atoms(h), qkv_half ? 2 * h->wg : h->wg));  // one activation box and weight slot per token tile
    if (h->tm) bb = 4 * (int)kTmChunkBytes;
    // + the epilogue staging area (the token-major epilogues store straight from registers)
    const int work = plans[i].a_cnt > 0 ? kAttnWork : bb + (h->tm ? 0 : 16 * 1024);
    // Attention CTAs keep their activation area inside the Q region (first 64 KB) so that the
    // prefix-K prefetch into the K/V area survives the GEMM stages in between.
    plans[i].b_bytes = plans[i].a_cnt > 0 ? std::max(tile, std::min(bb, 64 * 1024)) : bb;
    // ring slots of wg atoms: bf16 (wg x 16 KB) or E4M3 (wg x 8 KB)
    const int slot_bytes = h->fp8_stream ? h->wg * kAtomBytes / 2 : h->wg * kAtomBytes;
    plans[i].ring_slots = std::min(std::min(kMaxRing, h->ring_max), (kSmemUse - work) / slot_bytes);
    if (plans[i].ring_slots < 1) return fail(h, FA_ERR_INVALID, "shared-memory plan leaves no weight ring");
    // every unit's smallest activation batch (whole boxes and weight slots, all its token tiles)
    // must fit this CTA's activation area: the MMA lane never splits below that granule
    for (int m = 0; m < 4; ++m)
      for (const GemmUnit& x : per[i * 4 + m]) {
        const int aps = x.half ? 2 * h->wg : h->wg, gran = std::max(act_box_atoms(h), aps);
        const int nt = ntiles_of(m, x.grp);
        if (gran * nt * tile > plans[i].b_bytes)
          return fail(h, FA_ERR_INVALID, "plan error: a %d-atom activation batch of %d token tiles exceeds CTA %d's %d-byte area",
                      gran, nt, i, plans[i].b_bytes);
      }
    for (int m = 0; m < 4; ++m) {
      plans[i].g_off[m] = (int)gu.size();
      plans[i].g_cnt[m] = (int)per[i * 4 + m].size();
      gu.insert(gu.end(), per[i * 4 + m].begin(), per[i * 4 + m].end());
    }
  }
  if (h->tm)
    for (int i = 0; i < nblk; ++i)
      if (plans[i].b_bytes < 2 * (int)kTmChunkBytes || plans[i].ring_slots < 2)  // a 128-row chunk takes 2 ring slots
        return fail(h, FA_ERR_INVALID, "plan error: CTA %d has room for fewer than two activation chunks or ring slots", i);
  if (gu.size() > h->n_gunits_cap) {
    if (h->d_gunits) cudaFree(h->d_gunits);
    FA_CUDA(h, cudaMalloc(&h->d_gunits, gu.size() * sizeof(GemmUnit)));
    h->n_gunits_cap = gu.size();
  }
  if (au.size() > h->n_aunits_cap) {
    if (h->d_aunits) cudaFree(h->d_aunits);
    FA_CUDA(h, cudaMalloc(&h->d_aunits, au.size() * sizeof(AttnUnit)));
    h->n_aunits_cap = au.size();
  }
  FA_CUDA(h, cudaMemcpy(h->d_gunits, gu.data(), gu.size() * sizeof(GemmUnit), cudaMemcpyHostToDevice));
  FA_CUDA(h, cudaMemcpy(h->d_aunits, au.data(), au.size() * sizeof(AttnUnit), cudaMemcpyHostToDevice));
  FA_CUDA(h, cudaMemcpy(h->d_plans, plans.data(), plans.size() * sizeof(CtaPlan), cudaMemcpyHostToDevice));
  return FA_OK;
}

static fa_status build_params(fa_handle* h) {
  Params& p = h->params;
  memset(&p, 0, sizeof(p));
  const int L = h->cfg.num_layers, B = h->B;
  fa_status st;
  // weights: 3D boxes of wg K-atoms x 128 rows (one ring slot per load)
  if (h->fp8_stream) {  // E4M3 boxes of 128 K-values: wg / 2 per 128-row slot, wg per 64-row slot
#define MAPW8(i, base, K, rows, br, bn) if ((st = make_map3_u8(h, &p.maps[i], base, K, rows, br, bn)) != FA_OK) return st
    MAPW8(MAP_W_QKV, h->w8[0], D, (uint64_t)L * QKV_ROWS, 128, h->wg / 2);
    MAPW8(MAP_W_O, h->w8[1], QD, (uint64_t)L * D, 128, h->wg / 2);
    MAPW8(MAP_W_GU, h->w8[2], D, (uint64_t)L * 2 * F, 128, h->wg / 2);
    MAPW8(MAP_W_DN, h->w8[3], F, (uint64_t)L * D, 128, h->wg / 2);
    MAPW8(MAP_W_QKV_H, h->w8[0], D, (uint64_t)L * QKV_ROWS, 64, h->wg);
    MAPW8(MAP_W_GU_H, h->w8[2], D, (uint64_t)L * 2 * F, 64, h->wg);
#undef MAPW8
    for (int m = 0; m < 4; ++m) p.wscale[m] = h->ws8[m];
    const char* ea = getenv("FA_F8_AHEAD");
    p.f8_ahead = !(ea && atoi(ea) == 0);
  } else {
#define MAPW(i, base, K, rows) if ((st = make_map3(h, &p.maps[i], base, K, rows, 128, h->wg)) != FA_OK) return st
    MAPW(MAP_W_QKV, h->w_qkv, D, (uint64_t)L * QKV_ROWS);
    MAPW(MAP_W_O, h->w_o, QD, (uint64_t)L * D);
    MAPW(MAP_W_GU, h->w_gu, D, (uint64_t)L * 2 * F);
    MAPW(MAP_W_DN, h->w_dn, F, (uint64_t)L * D);
#undef MAPW
    // half-row units: 64-row boxes of 2 x wg atoms (one ring slot)
    if ((st = make_map3(h, &p.maps[MAP_W_QKV_H], h->w_qkv, D, (uint64_t)L * QKV_ROWS, 64, 2 * h->wg)) != FA_OK) return st;
    if ((st = make_map3(h, &p.maps[MAP_W_GU_H], h->w_gu, D, (uint64_t)L * 2 * F, 64, 2 * h->wg)) != FA_OK) return st;
  }
  const uint32_t ba = (uint32_t)act_box_atoms(h);
#define MAP3(i, base, K, rows, br, bat) if ((st = make_map3(h, &p.maps[i], base, K, rows, br, bat)) != FA_OK) return st
  MAP3(MAP_XN, h->xn, D, h->NPAD, h->NTILE, ba);
  MAP3(MAP_ATTN, h->attn, QD, h->NPAD, h->NTILE, ba);
  MAP3(MAP_H, h->hbuf, F, h->NPAD, h->NTILE, ba);
  MAP3(MAP_Q, h->q, HD, (uint64_t)B * H * TPAD, 128, 4);
  MAP3(MAP_K, h->kcache, HD, (uint64_t)B * L * h->LPAD, 128, 4);
  MAP3(MAP_VT, h->vtcache, h->LPAD, (uint64_t)B * L * HD, 128, 2);
  MAP3(MAP_SK, h->sk, HD, (uint64_t)B * TPAD, 64, 4);
  MAP3(MAP_SVT, h->svt, TPAD, (uint64_t)B * HD, 128, 1);
#undef MAP3
  p.box_atoms = (int)ba;
  p.wg = h->wg;
  p.L = L; p.T = h->cfg.horizon; p.B = B; p.NT = h->NT; p.NPAD = h->NPAD; p.NTILE = h->NTILE; p.TG = h->TG;
  for (int m = 0; m < 4; ++m) p.tg[m] = h->tgm[m];
  p.ngroups = h->ngroups; p.nsteps = h->cfg.num_steps; p.LPAD = h->LPAD; p.AD = h->cfg.action_dim;
  p.split_o = h->split_o_eff; p.split_dn = h->split_dn_eff;
  p.attn_whole = h->attn_whole ? 1 : 0;
  p.dt = -1.0f / (float)h->cfg.num_steps;
  p.invT = 1.0f / (float)h->cfg.horizon;
  p.gunits = h->d_gunits; p.aunits = h->d_aunits; p.plans = h->d_plans;
  p.valid_len = h->d_valid; p.nchunks = h->d_nchunks;
  p.mods = h->mods; p.mod_final = h->mod_final; p.rope_cos = h->rope_cos; p.rope_sin = h->rope_sin;
  p.w_ain = h->w_ain; p.b_ain = h->b_ain; p.w_aout = h->w_aout; p.b_aout = h->b_aout;
  p.x_t = h->x_t; p.x = h->x; p.part = h->part; p.xn = h->xn; p.attn = h->attn; p.hbuf = h->hbuf;
  p.q = h->q; p.sk = h->sk; p.svt = h->svt; p.opart = h->opart; p.oml = h->oml;
  p.bar = h->ctrl; p.err = reinterpret_cast<int*>(h->ctrl + 1);
  p.stage_ns = nullptr;
  p.inject_barrier = -1;
  p.trace = h->trace;
  p.trace_step = h->trace_step;
  p.trace_layer = h->trace_layer;
  p.spin_limit = 1u << 24;
  p.l2_ahead = l2_ahead_layers();
  {
    const int K4[4] = {D, QD, D, F};
    const void* w16[4] = {h->w_qkv, h->w_o, h->w_gu, h->w_dn};
    for (int m = 0; m < 4; ++m) {
      p.wraw[m] = reinterpret_cast<const uint8_t*>(h->fp8_stream ? h->w8[m] : w16[m]);
      p.wrow_bytes[m] = h->fp8_stream ? K4[m] : 2 * K4[m];
    }
  }
  return FA_OK;
}

static fa_status bind_impl(fa_handle* h, int batch, const void* k, const void* v, int src_rows, const int* valid_len,
                           fa_kv_layout layout, fa_stream stream, const int* rowmap);

extern "C" fa_status fa_bind_prefix_kv(fa_handle* h, int batch, const void* k, const void* v, int src_rows,
                                       const int* valid_len, fa_kv_layout layout, fa_stream stream) {
  if (!h) return fail(h, FA_ERR_INVALID, "null handle");
  return bind_impl(h, batch, k, v, src_rows, valid_len, layout, stream, nullptr);
}

extern "C" fa_status fa_bind_prefix_kv_masked(fa_handle* h, int batch, const void* k, const void* v, int src_rows,
                                              const unsigned char* keep, fa_kv_layout layout, fa_stream stream) {
  if (!h) return fail(h, FA_ERR_INVALID, "null handle");
  if (batch < 1 || batch > h->cfg.max_batch) return fail(h, FA_ERR_INVALID, "batch %d outside 1..%d", batch, h->cfg.max_batch);
  FA_CUDA(h, cudaSetDevice(h->device));
  std::vector<int> counts;
  fa_status st = masked_rows(h, batch, src_rows, keep, reinterpret_cast<cudaStream_t>(stream), counts);
  if (st != FA_OK) return st;
  return bind_impl(h, batch, k, v, src_rows, counts.data(), layout, stream, h->d_rowmap);
}

static fa_status bind_impl(fa_handle* h, int batch, const void* k, const void* v, int src_rows, const int* valid_len,
                           fa_kv_layout layout, fa_stream stream, const int* rowmap) {
  if (h->kind == FA_MODEL_MOLMOACT2)
    return ma2_bind(h, batch, k, v, src_rows, valid_len, reinterpret_cast<cudaStream_t>(stream), rowmap);
  if (batch < 1 || batch > h->cfg.max_batch) return fail(h, FA_ERR_INVALID, "batch %d outside 1..%d", batch, h->cfg.max_batch);
  if (!valid_len) return fail(h, FA_ERR_INVALID, "valid_len is null");
  if (layout != FA_KV_COMPACT_SPLIT_HALF && layout != FA_KV_FLASHRT_INTERLEAVED) return fail(h, FA_ERR_INVALID, "unknown kv layout");
  int maxvl = 0;
  for (int b = 0; b < batch; ++b) {
    if (valid_len[b] < 0 || valid_len[b] > src_rows || valid_len[b] > h->cfg.max_prefix)
      return fail(h, FA_ERR_INVALID, "valid_len[%d]=%d outside 0..min(src_rows=%d, max_prefix=%d)", b, valid_len[b], src_rows,
                  h->cfg.max_prefix);
    maxvl = std::max(maxvl, valid_len[b]);
  }
  if (maxvl > 0 && (!k || !v)) return fail(h, FA_ERR_INVALID, "k/v pointers are null");
  if (maxvl > 0 && (!is_device_ptr(k) || !is_device_ptr(v))) return fail(h, FA_ERR_INVALID, "k/v must be device pointers");
  FA_CUDA(h, cudaSetDevice(h->device));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int L_ = h->cfg.num_layers;
  if (h->kv_ready && !rowmap && batch == h->B && (int)h->valid_len.size() == batch &&
      std::equal(valid_len, valid_len + batch, h->valid_len.begin())) {
    // Same batch and valid lengths: the work plan, tensor maps, valid lengths and RoPE tables on the
    // device all stay; only the cache contents are rewritten, asynchronously on `stream` (ordered
    // after earlier launches on that stream, like the reference's in-launch KV handoff,
    // src/pi05/mk6.cu:258-277).
    const int sr = std::max(src_rows, 1);
    bind_k_kernel<<<dim3(std::max(1, h->LPAD * HD / 256 / 4), L_, batch), 256, 0, s>>>(
        (const bf16*)k, sr, h->d_valid, nullptr, L_, h->LPAD, layout == FA_KV_FLASHRT_INTERLEAVED, h->kcache);
    FA_CUDA(h, cudaGetLastError());
    bind_vt_kernel<<<dim3(h->LPAD / 32, HD / 32, batch * L_), dim3(32, 8), 0, s>>>((const bf16*)v, sr, h->d_valid, nullptr,
                                                                                 L_, h->LPAD, h->vtcache);
    FA_CUDA(h, cudaGetLastError());
    return FA_OK;
  }
  FA_CUDA(h, cudaStreamSynchronize(s));  // previous launches may still read the cache and plan
  const int T = h->cfg.horizon, L = h->cfg.num_layers;
  h->B = batch;
  h->NT = batch * T;
  h->NTILE = h->NT <= 64 ? 64 : 128;
  if (const char* e = getenv("FA_NTILE"); e && atoi(e) == 64) h->NTILE = 64;  // tuning knob
  h->NPAD = round_up(h->NT, h->NTILE);
  h->TG = 256 / h->NTILE;
  h->ngroups = (h->NPAD / h->NTILE + h->TG - 1) / h->TG;
  h->LPAD = std::max(KCH, round_up(h->cfg.max_prefix, KCH));
  h->valid_len.assign(valid_len, valid_len + batch);
  std::vector<int> nch(batch);
  for (int b = 0; b < batch; ++b) nch[b] = (valid_len[b] + KCH - 1) / KCH;
  FA_CUDA(h, cudaMemcpy(h->d_valid, valid_len, batch * sizeof(int), cudaMemcpyHostToDevice));
  FA_CUDA(h, cudaMemcpy(h->d_nchunks, nch.data(), batch * sizeof(int), cudaMemcpyHostToDevice));
  fa_status st;
  if ((st = build_plan(h)) != FA_OK) return st;
  if ((st = build_params(h)) != FA_OK) return st;
  const int sr = std::max(src_rows, 1);
  bind_k_kernel<<<dim3(std::max(1, h->LPAD * HD / 256 / 4), L, batch), 256, 0, s>>>(
      (const bf16*)k, sr, h->d_valid, rowmap, L, h->LPAD, layout == FA_KV_FLASHRT_INTERLEAVED, h->kcache);
  FA_CUDA(h, cudaGetLastError());
  bind_vt_kernel<<<dim3(h->LPAD / 32, HD / 32, batch * L), dim3(32, 8), 0, s>>>((const bf16*)v, sr, h->d_valid, rowmap, L,
                                                                              h->LPAD, h->vtcache);
  FA_CUDA(h, cudaGetLastError());
  rope_kernel<<<64, 256, 0, s>>>(h->d_valid, batch, T, h->rope_cos, h->rope_sin);
  FA_CUDA(h, cudaGetLastError());
  FA_CUDA(h, cudaStreamSynchronize(s));
  h->kv_ready = true;
  return FA_OK;
}

extern "C" fa_status fa_set_stage_timing(fa_handle* h, int enable) {
  if (!h) return FA_ERR_INVALID;
  h->timing = enable != 0;
  return FA_OK;
}

extern "C" fa_status fa_get_stage_cycles(fa_handle* h, uint64_t* out, int n) {
  if (!h || !out) return fail(h, FA_ERR_INVALID, "null argument");
  FA_CUDA(h, cudaSetDevice(h->device));
  if (is_device_ptr(out)) {  // device destination: copied on the last launch's stream, no host synchronisation
    const int m = std::max(0, std::min(n, (int)kMaxStages));
    if (m > 0) FA_CUDA(h, cudaMemcpyAsync(out, h->stage_ns, (size_t)m * 8, cudaMemcpyDeviceToDevice, h->last_stream));
    return FA_OK;
  }
  unsigned long long tmp[kMaxStages];
  FA_CUDA(h, cudaMemcpy(tmp, h->stage_ns, sizeof(tmp), cudaMemcpyDeviceToHost));
  for (int i = 0; i < n; ++i) out[i] = i < kMaxStages ? tmp[i] : 0;
  return FA_OK;
}

extern "C" fa_status fa_sample_actions(fa_handle* h, int batch, const float* noise, float* actions_out, fa_stream stream) {
  if (!h || !noise || !actions_out) return fail(h, FA_ERR_INVALID, "null argument");
  if (h->kind == FA_MODEL_MOLMOACT2) return ma2_sample(h, batch, noise, actions_out, reinterpret_cast<cudaStream_t>(stream));
  if (!h->weights_ready) return fail(h, FA_ERR_STATE, "weights not loaded");
  if (!h->kv_ready) return fail(h, FA_ERR_STATE, "prefix KV not bound");
  if (batch != h->B) return fail(h, FA_ERR_INVALID, "batch %d differs from the bound batch %d", batch, h->B);
  FA_CUDA(h, cudaSetDevice(h->device));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t bytes = (size_t)h->NT * h->cfg.action_dim * sizeof(float);
  Params& p = h->params;
  p.stage_ns = h->timing ? h->stage_ns : nullptr;
  FA_CUDA(h, cudaMemsetAsync(h->ctrl, 0, kCtrlWords * sizeof(unsigned int), s));
  if (h->timing) FA_CUDA(h, cudaMemsetAsync(h->stage_ns, 0, NUM_STAGES * sizeof(unsigned long long), s));
  FA_CUDA(h, cudaMemcpyAsync(h->x_t, noise, bytes, cudaMemcpyDefault, s));
  void* args[] = {&p};
  const void* kern = h->fp8_stream ? (const void*)fa::pi05::pi05_denoise_kernel_f8
                     : h->tm       ? (const void*)fa::pi05::pi05_denoise_kernel_tm
                                   : (const void*)fa::pi05::pi05_denoise_kernel;
  FA_CUDA(h, cudaLaunchCooperativeKernel(kern, dim3(h->num_sms), dim3(kThreads), args, kSmemDyn, s));
  FA_CUDA(h, cudaMemcpyAsync(actions_out, h->x_t, bytes, cudaMemcpyDefault, s));
  h->last_launches = 1;
  h->last_stream = s;
  return FA_OK;
}

extern "C" fa_status fa_sync(fa_handle* h, fa_stream stream) {
  if (!h) return FA_ERR_INVALID;
  FA_CUDA(h, cudaSetDevice(h->device));
  FA_CUDA(h, cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
  unsigned int ctrl[2];
  FA_CUDA(h, cudaMemcpy(ctrl, h->ctrl, sizeof(ctrl), cudaMemcpyDeviceToHost));
  if (ctrl[1] != 0)
    return fail(h, FA_ERR_TIMEOUT, "in-kernel wait ran out (code %u; %u grid-barrier arrivals, %u CTAs)", ctrl[1], ctrl[0],
                (unsigned)h->num_sms);
  return FA_OK;
}

// Diagnostics: arm (step >= 0) or read back (step < 0) a clock64 trace of one (step, layer).
extern "C" fa_status fa_debug_trace(fa_handle* h, int step, int layer, unsigned long long* host_out, int n) {
  if (!h) return FA_ERR_INVALID;
#ifndef FA_TRACE
  (void)step; (void)layer; (void)host_out; (void)n;
  return fail(h, FA_ERR_UNSUPPORTED, "stage tracing is compiled in only by a -DFA_TRACE build");
#endif
  const size_t need = (size_t)kMaxStages * h->num_sms * kTrStride;
  FA_CUDA(h, cudaSetDevice(h->device));
  if (step < 0) {
    if (!h->trace) return fail(h, FA_ERR_STATE, "trace not armed");
    FA_CUDA(h, cudaMemcpy(host_out, h->trace, std::min((size_t)std::max(n, 0), need) * 8, cudaMemcpyDeviceToHost));
    return FA_OK;
  }
  if (!h->trace) {
    fa_status st = dalloc(h, &h->trace, need);
    if (st != FA_OK) return st;
  }
  FA_CUDA(h, cudaMemset(h->trace, 0, need * 8));
  h->trace_step = h->params.trace_step = step;
  h->trace_layer = h->params.trace_layer = layer;
  h->params.trace = h->trace;
  ma2_set_debug(h);
  return FA_OK;
}

extern "C" fa_status fa_set_fault_injection(fa_handle* h, int barrier_index, unsigned int spin_limit) {
  if (!h) return FA_ERR_INVALID;
  h->params.inject_barrier = barrier_index;
  h->params.spin_limit = spin_limit ? spin_limit : (1u << 24);
  ma2_set_debug(h);
  return FA_OK;
}

// ------------------------------------------------------------------ allocation-free conditioning
// Some callers cannot allocate device memory when they need the adaRMS modulations: a robot
// control process that pins its memory budget after start-up, or a host that owns a fixed pool
// and forbids cudaMalloc outside it. For them, fa_pi05_modulations_noalloc computes the same
// time embedding -> conditioning MLP -> per-layer modulations as fa_pi05_load_weights, but its
// scratch (embedding, MLP hidden and conditioning vectors) lives in this file-scope array,
// sized for at most kNoAllocMaxSteps Euler steps of width 1024 (3 x 50 x 1024 floats = 600 KB,
// held by every GPU that loads this library until the process exits).
constexpr int kNoAllocMaxSteps = 50;
static __device__ __align__(256) float g_cond_scratch[3 * kNoAllocMaxSteps * D];

// Device address of g_cond_scratch on the current device. The host-side symbol is only a
// stand-in and must never be handed to a kernel. The lookup is repeated on every call (a host-side
// table lookup once the module is loaded), so the address stays right after a cudaDeviceReset,
// which reloads the module at a new address.
static fa_status cond_scratch_address(float** out) {
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_cond_scratch);
  if (e != cudaSuccess)
    return fail(nullptr, FA_ERR_CUDA, "cudaGetSymbolAddress(g_cond_scratch): %s", cudaGetErrorString(e));
  *out = reinterpret_cast<float*>(ptr);
  return FA_OK;
}

// True when `p` is device (or managed) memory that kernels on `device` may use directly.
static bool on_device(const void* p, int device) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (a.type == cudaMemoryTypeManaged) return true;
  return a.type == cudaMemoryTypeDevice && a.device == device;
}

extern "C" fa_status fa_pi05_modulations_noalloc(const fa_pi05_weights* w, int num_layers, int num_steps,
                                                 float* mods_out, float* mod_final_out, fa_stream stream) {
  if (!w || !mods_out || !mod_final_out) return fail(nullptr, FA_ERR_INVALID, "null argument");
  if (num_steps < 1 || num_steps > kNoAllocMaxSteps)
    return fail(nullptr, FA_ERR_INVALID, "num_steps %d outside 1..%d (the static scratch holds %d steps)", num_steps,
                kNoAllocMaxSteps, kNoAllocMaxSteps);
  if (num_layers < 1 || num_layers > 64) return fail(nullptr, FA_ERR_INVALID, "num_layers %d outside 1..64", num_layers);
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return fail(nullptr, FA_ERR_CUDA, "cudaGetDevice failed");
  // An error left pending by the caller's earlier work would otherwise be reported (and cleared)
  // as if one of these launches had failed: refuse to start instead and leave it in place.
  const cudaError_t pending = cudaPeekAtLastError();
  if (pending != cudaSuccess)
    return fail(nullptr, FA_ERR_CUDA, "a CUDA error is pending from earlier work on this thread: %s",
                cudaGetErrorString(pending));
  const fa_tensor* need[] = {&w->ln_in_w, &w->ln_in_b, &w->ln_post_w, &w->ln_post_b, &w->norm_w,
                             &w->norm_b, &w->time_in_w, &w->time_in_b, &w->time_out_w, &w->time_out_b};
  for (const fa_tensor* t : need) {
    if (!t->ptr || !on_device(t->ptr, device))
      return fail(nullptr, FA_ERR_INVALID,
                  "every conditioning weight must be memory of the current device %d (none is staged here)", device);
    if (t->dtype != FA_DT_F32 && t->dtype != FA_DT_BF16 && t->dtype != FA_DT_F16)
      return fail(nullptr, FA_ERR_INVALID, "unsupported weight dtype %d", (int)t->dtype);
  }
  if (!on_device(mods_out, device) || !on_device(mod_final_out, device))
    return fail(nullptr, FA_ERR_INVALID, "mods_out / mod_final_out must be memory of the current device %d", device);
  float* scratch = nullptr;
  fa_status st = cond_scratch_address(&scratch);
  if (st != FA_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int S = num_steps, L = num_layers;
  float* emb = scratch;                   // [S][1024]; every element is written before it is read,
  float* h1 = scratch + (size_t)S * D;    // so nothing from an earlier call needs clearing
  float* cond = scratch + (size_t)2 * S * D;
  const size_t smem = (size_t)S * D * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(linear_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return fail(nullptr, FA_ERR_CUDA, "cannot reserve %zu bytes of shared memory", smem);
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms < 1)
    return fail(nullptr, FA_ERR_CUDA, "cudaDeviceGetAttribute(multiProcessorCount) failed on device %d", device);
  const int grid = sms * 2;
  // every launch is checked at once: nothing was pending on entry, so an error here is ours
#define NOALLOC_CHECK(what)                                                                        \
  do {                                                                                             \
    const cudaError_t e_ = cudaGetLastError();                                                     \
    if (e_ != cudaSuccess) return fail(nullptr, FA_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e_)); \
  } while (0)
  time_embed_kernel<<<8, 256, 0, s>>>(emb, S, D);
  NOALLOC_CHECK("time embedding");
  linear_f32_kernel<<<grid, 256, smem, s>>>(w->time_in_w.ptr, w->time_in_w.dtype, w->time_in_b.ptr, w->time_in_b.dtype,
                                            emb, S, D, D, h1, D, 1);
  NOALLOC_CHECK("time MLP in");
  linear_f32_kernel<<<grid, 256, smem, s>>>(w->time_out_w.ptr, w->time_out_w.dtype, w->time_out_b.ptr,
                                            w->time_out_b.dtype, h1, S, D, D, cond, D, 1);
  NOALLOC_CHECK("time MLP out");
  const size_t sstride = (size_t)L * 2 * MOD;
  for (int l = 0; l < L; ++l) {
    linear_f32_kernel<<<grid, 256, smem, s>>>(
        (const char*)w->ln_in_w.ptr + (size_t)l * MOD * D * dtype_size(w->ln_in_w.dtype), w->ln_in_w.dtype,
        (const char*)w->ln_in_b.ptr + (size_t)l * MOD * dtype_size(w->ln_in_b.dtype), w->ln_in_b.dtype, cond, S, D, MOD,
        mods_out + (size_t)l * 2 * MOD, sstride, 0);
    NOALLOC_CHECK("input adaRMS dense");
    linear_f32_kernel<<<grid, 256, smem, s>>>(
        (const char*)w->ln_post_w.ptr + (size_t)l * MOD * D * dtype_size(w->ln_post_w.dtype), w->ln_post_w.dtype,
        (const char*)w->ln_post_b.ptr + (size_t)l * MOD * dtype_size(w->ln_post_b.dtype), w->ln_post_b.dtype, cond, S, D,
        MOD, mods_out + (size_t)l * 2 * MOD + MOD, sstride, 0);
    NOALLOC_CHECK("post-attention adaRMS dense");
  }
  linear_f32_kernel<<<grid, 256, smem, s>>>(w->norm_w.ptr, w->norm_w.dtype, w->norm_b.ptr,
                                            w->norm_b.dtype, cond, S, D, MOD, mod_final_out, MOD, 0);
  NOALLOC_CHECK("final adaRMS dense");
#undef NOALLOC_CHECK
  return FA_OK;
}
