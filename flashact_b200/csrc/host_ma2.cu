// Host side of the MolmoAct2 engine behind the C ABI: buffers, weight packing, context bind,
// work planning, TMA descriptors and launch of fa::ma2::ma2_denoise_kernel.
#include "fa_ma2.cuh"
#include "host_common.cuh"

namespace fa {
namespace ma2 {
__global__ void ma2_denoise_kernel(const __grid_constant__ Params p);
__global__ void ma2_denoise_kernel_tm(const __grid_constant__ Params p);
}
}  // namespace fa

namespace M = fa::ma2;

struct Ma2State {
  M::Params params;
  bf16* w[M::NUM_MATS] = {};
  float* bias[M::NUM_MATS] = {};
  float* b_up = nullptr;
  float *mods = nullptr, *mod_final = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
  float *w_ain = nullptr, *b_ain = nullptr, *w_aout = nullptr, *b_aout = nullptr;
  float *x_t = nullptr, *x = nullptr, *part = nullptr, *oml = nullptr;
  bf16 *xn = nullptr, *qkv = nullptr, *sattn = nullptr, *cattn = nullptr, *hbuf = nullptr;
  bf16 *opart = nullptr, *kctx = nullptr, *vctx = nullptr, *aout_bf16 = nullptr;
  int* d_ctx = nullptr;
  GemmUnit* d_gunits = nullptr;
  AttnUnit* d_aunits = nullptr;
  CtaPlan* d_plans = nullptr;
  size_t gcap = 0, acap = 0;
  int B = 0, NT = 0, NPAD = 0, NTILE = 64, TG = 4, ngroups = 1, LKPAD = 0, adim = 0;
  int self_q = 8;
  bool cross_whole = false;
  bool tm = false;  // token-major GEMMs (bound batch = one tile of <= 64 tokens)
  int wg = 4;  // weight atoms per ring slot
  int ba = 4;  // activation atoms per TMA box
  int split[M::NUM_MATS] = {1, 3, 3, 3, 1, 6};
  int split_eff[M::NUM_MATS] = {1, 3, 3, 3, 1, 6};  // K-splits used for the bound batch
  std::vector<int> ctx;
  bool weights = false, mods_set = false, bound = false;
};

static constexpr int kMatRows[M::NUM_MATS] = {M::QKV_ROWS, M::D, M::D, M::D, 2 * M::F, M::D};
static constexpr int kMatK[M::NUM_MATS] = {M::D, M::D, M::D, M::D, M::D, M::F};

// Context bind: dst[b][l][r][:] = src[b][l][map(r)][:] for r < len[b] (map = identity, or the
// kept rows of a masked bind), zero up to LKPAD.
static __global__ void ma2_bind_ctx_kernel(const bf16* src, int src_rows, const int* len, const int* rowmap, int L,
                                           int LKPAD, bf16* dst) {
  const int b = blockIdx.z, l = blockIdx.y;
  const int n = len[b];
  const size_t per = (size_t)LKPAD * M::D / 8;  // 16-byte pieces
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < per; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / (M::D / 8)), seg = (int)(i % (M::D / 8));
    uint4 val = make_uint4(0, 0, 0, 0);
    const int sr = rowmap && r < n ? rowmap[(size_t)b * src_rows + r] : r;
    if (r < n) val = *reinterpret_cast<const uint4*>(src + (((size_t)b * L + l) * src_rows + sr) * M::D + seg * 8);
    *reinterpret_cast<uint4*>(dst + (((size_t)b * L + l) * LKPAD + r) * M::D + seg * 8) = val;
  }
}

// V^T bind: dst[b][l][d][r] = src[b][l][map(r)][d] for r < len[b], zero up to LKPAD (32 x 32 tiles
// through shared memory).
static __global__ void ma2_bind_vt_kernel(const bf16* src, int src_rows, const int* len, const int* rowmap, int L,
                                          int LKPAD, bf16* dst) {
  __shared__ bf16 tile[32][33];
  const int b = blockIdx.z / L, l = blockIdx.z % L;
  const int n = len[b];
  const int r0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, d = d0 + threadIdx.x;
    const int sr = rowmap && r < n ? rowmap[(size_t)b * src_rows + r] : r;
    tile[i][threadIdx.x] = r < n ? src[(((size_t)b * L + l) * src_rows + sr) * M::D + d] : __float2bfloat16(0.f);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int d = d0 + i, r = r0 + threadIdx.x;
    dst[(((size_t)b * L + l) * M::D + d) * LKPAD + r] = tile[threadIdx.x][i];
  }
}

fa_status ma2_create(const fa_config& c, int device, fa_handle* h) {
  if (c.width != M::D || c.num_heads != M::H || c.num_kv_heads != M::H || c.head_dim != M::HD || c.mlp_dim != M::F)
    return fail(h, FA_ERR_INVALID, "MolmoAct2 expert geometry must be width 768, 8 heads, 8 kv heads, head_dim 96, mlp 3072");
  if (c.num_layers < 1 || c.num_layers > 64 || c.horizon < 1 || c.horizon > M::TMAX || c.action_dim < 1 ||
      c.action_dim > 32 || c.valid_action_dim < 0 || c.valid_action_dim > c.action_dim || c.max_prefix < 1 ||
      c.max_prefix > M::MAX_CH * M::KC || c.max_batch < 1 || c.max_batch > 256 || c.num_steps < 1 || c.num_steps > 50)
    return fail(h, FA_ERR_INVALID,
                "config out of range (layers 1..64, horizon 1..32, action_dim 1..32, context 1..4096, batch 1..256, steps 1..50)");
  if (cudaSetDevice(device) != cudaSuccess) return fail(h, FA_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  Ma2State* s = new Ma2State();
  h->ma2 = s;
  // Tuning knob: FA_MA2_SPLITS="qkv,so,cq,co,gu,dn" K-split factors (each must divide the
  // matrix's K atoms: 12 for the 768-wide inputs, 48 for down; qkv and gu stay 1 -- their
  // epilogues need whole sums).
  if (const char* e = getenv("FA_MA2_SPLITS")) {
    int v[M::NUM_MATS];
    if (sscanf(e, "%d,%d,%d,%d,%d,%d", &v[0], &v[1], &v[2], &v[3], &v[4], &v[5]) == M::NUM_MATS)
      for (int m = 0; m < M::NUM_MATS; ++m)
        if (v[m] >= 1 && (kMatK[m] / 64) % v[m] == 0 && (m != M::MAT_QKV && m != M::MAT_GU ? true : v[m] == 1))
          s->split[m] = v[m];
  }
  s->adim = c.valid_action_dim > 0 ? c.valid_action_dim : c.action_dim;
  const int L = c.num_layers, S = c.num_steps, MB = c.max_batch;
  const int NPADm = round_up(MB * c.horizon, 128);
  const int LKm = round_up(c.max_prefix, M::KC);
  fa_status st = FA_OK;
#define ALLOC(ptr, n) if ((st = dalloc(h, &(ptr), (size_t)(n))) != FA_OK) return st
  for (int m = 0; m < M::NUM_MATS; ++m) {
    ALLOC(s->w[m], (size_t)L * kMatRows[m] * kMatK[m]);
    ALLOC(s->bias[m], (size_t)L * (m == M::MAT_GU ? M::F : kMatRows[m]));
  }
  ALLOC(s->b_up, (size_t)L * M::F);
  ALLOC(s->mods, (size_t)S * L * 9 * M::D);
  ALLOC(s->mod_final, (size_t)S * 2 * M::D);
  ALLOC(s->rope_cos, M::TMAX * 48);
  ALLOC(s->rope_sin, M::TMAX * 48);
  ALLOC(s->w_ain, (size_t)M::D * c.action_dim);
  ALLOC(s->b_ain, M::D);
  ALLOC(s->w_aout, (size_t)c.action_dim * M::D);
  ALLOC(s->aout_bf16, (size_t)c.action_dim * M::D);
  ALLOC(s->b_aout, c.action_dim);
  ALLOC(s->x_t, (size_t)NPADm * c.action_dim);
  ALLOC(s->x, (size_t)NPADm * M::D);
  ALLOC(s->part, (size_t)12 * NPADm * M::D);
  ALLOC(s->xn, (size_t)NPADm * M::D);
  ALLOC(s->qkv, (size_t)NPADm * M::QKV_ROWS);
  ALLOC(s->sattn, (size_t)NPADm * M::D);
  ALLOC(s->cattn, (size_t)NPADm * M::D);
  ALLOC(s->hbuf, (size_t)NPADm * M::F);
  ALLOC(s->opart, (size_t)MB * M::H * M::MAX_CH * M::TMAX * M::HD);
  ALLOC(s->oml, (size_t)MB * M::H * M::MAX_CH * M::TMAX * 2);
  ALLOC(s->kctx, (size_t)MB * L * LKm * M::D);
  ALLOC(s->vctx, (size_t)MB * L * LKm * M::D);
  ALLOC(s->d_ctx, MB);
  ALLOC(s->d_plans, h->num_sms);
  ALLOC(h->ctrl, fa::kCtrlWords);
  ALLOC(h->stage_ns, fa::kMaxStages);
#undef ALLOC
  // default RoPE tables: theta 10000 over the 96 head dims, positions 0..T-1
  std::vector<float> cs(M::TMAX * 48, 0.f), sn(M::TMAX * 48, 0.f);
  for (int t = 0; t < M::TMAX; ++t)
    for (int i = 0; i < 48; ++i) {
      const float inv = (float)(1.0 / pow(10000.0, (double)(2 * i) / M::HD));
      const float ang = (float)t * inv;
      cs[t * 48 + i] = (float)cos((double)ang);
      sn[t * 48 + i] = (float)sin((double)ang);
    }
  FA_CUDA(h, cudaMemcpy(s->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  FA_CUDA(h, cudaMemcpy(s->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  for (const void* k : {(const void*)M::ma2_denoise_kernel, (const void*)M::ma2_denoise_kernel_tm}) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::kSmemDyn) != cudaSuccess)
      return fail(h, FA_ERR_CUDA, "cannot reserve %d bytes of shared memory", fa::kSmemDyn);
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, fa::kThreads, fa::kSmemDyn) != cudaSuccess || occ < 1)
      return fail(h, FA_ERR_UNSUPPORTED, "megakernel does not fit on an SM (occupancy %d)", occ);
  }
  return FA_OK;
}

void ma2_destroy(fa_handle* h) {
  if (h && h->ma2) {
    delete h->ma2;
    h->ma2 = nullptr;
  }
}

extern "C" fa_status fa_ma2_load_weights(fa_handle* h, const fa_ma2_weights* w) {
  if (!h || !w) return fail(h, FA_ERR_INVALID, "null argument");
  if (h->kind != FA_MODEL_MOLMOACT2 || !h->ma2) return fail(h, FA_ERR_INVALID, "not a MolmoAct2 handle");
  Ma2State* s = h->ma2;
  FA_CUDA(h, cudaSetDevice(h->device));
  const int L = h->cfg.num_layers, AD = h->cfg.action_dim;
  std::vector<void*> tmp;
  struct Cleanup {
    std::vector<void*>& t;
    ~Cleanup() { for (void* p : t) cudaFree(p); }
  } cleanup{tmp};
  fa_status st;
  const fa_tensor* mats[M::NUM_MATS] = {&w->w_qkv, &w->w_so, &w->w_cq, &w->w_co, &w->w_gate, &w->w_down};
  const fa_tensor* biases[M::NUM_MATS] = {&w->b_qkv, &w->b_so, &w->b_cq, &w->b_co, &w->b_gate, &w->b_down};
  const char* names[M::NUM_MATS] = {"w_qkv", "w_so", "w_cq", "w_co", "w_gate", "w_down"};
  for (int m = 0; m < M::NUM_MATS; ++m) {
    const int rows = m == M::MAT_GU ? M::F : kMatRows[m];
    const void *dw = nullptr, *db = nullptr;
    if ((st = stage_tensor(h, *mats[m], (size_t)L * rows * kMatK[m], names[m], &dw, tmp)) != FA_OK) return st;
    if ((st = stage_tensor(h, *biases[m], (size_t)L * rows, names[m], &db, tmp)) != FA_OK) return st;
    to_f32_kernel<<<64, 256>>>(db, biases[m]->dtype, s->bias[m], (size_t)L * rows);
    if (m == M::MAT_GU) {
      const void *du = nullptr, *dub = nullptr;
      if ((st = stage_tensor(h, w->w_up, (size_t)L * M::F * M::D, "w_up", &du, tmp)) != FA_OK) return st;
      if ((st = stage_tensor(h, w->b_up, (size_t)L * M::F, "b_up", &dub, tmp)) != FA_OK) return st;
      to_f32_kernel<<<64, 256>>>(dub, w->b_up.dtype, s->b_up, (size_t)L * M::F);
      // gate/up rows: tile mt, row 32 q + lane -> feature 64 mt + 16 q + (lane & 15); lanes < 16 gate
      std::vector<int2> map(2 * M::F);
      for (int mt = 0; mt < 2 * M::F / 128; ++mt)
        for (int r = 0; r < 128; ++r) {
          const int qd = r >> 5, lane = r & 31;
          map[mt * 128 + r] = make_int2(lane < 16 ? 0 : 1, 64 * mt + 16 * qd + (lane & 15));
        }
      PackSrc src = {{dw, du, du}, {mats[m]->dtype, w->w_up.dtype, w->w_up.dtype}, {M::F, M::F, M::F}};
      if ((st = pack_matrix(h, map, src, s->w[m], M::D, tmp)) != FA_OK) return st;
    } else {
      std::vector<int2> map(rows);
      for (int r = 0; r < rows; ++r) map[r] = make_int2(0, r);
      PackSrc src = {{dw, dw, dw}, {mats[m]->dtype, mats[m]->dtype, mats[m]->dtype}, {rows, rows, rows}};
      if ((st = pack_matrix(h, map, src, s->w[m], kMatK[m], tmp)) != FA_OK) return st;
    }
  }
  const void *aiw = nullptr, *aib = nullptr, *aow = nullptr, *aob = nullptr;
  if ((st = stage_tensor(h, w->ain_w, (size_t)M::D * AD, "ain_w", &aiw, tmp)) != FA_OK) return st;
  if ((st = stage_tensor(h, w->ain_b, M::D, "ain_b", &aib, tmp)) != FA_OK) return st;
  if ((st = stage_tensor(h, w->aout_w, (size_t)AD * M::D, "aout_w", &aow, tmp)) != FA_OK) return st;
  if ((st = stage_tensor(h, w->aout_b, AD, "aout_b", &aob, tmp)) != FA_OK) return st;
  to_f32_kernel<<<64, 256>>>(aiw, w->ain_w.dtype, s->w_ain, (size_t)M::D * AD);
  to_f32_kernel<<<4, 256>>>(aib, w->ain_b.dtype, s->b_ain, M::D);
  {  // the velocity head is applied with bf16 weights, as in the reference (mk_ma2.cu:44, :569)
    std::vector<int2> map(AD);
    for (int r = 0; r < AD; ++r) map[r] = make_int2(0, r);
    PackSrc src = {{aow, aow, aow}, {w->aout_w.dtype, w->aout_w.dtype, w->aout_w.dtype}, {AD, AD, AD}};
    const int saved = h->cfg.num_layers;
    h->cfg.num_layers = 1;
    st = pack_matrix(h, map, src, s->aout_bf16, M::D, tmp);
    h->cfg.num_layers = saved;
    if (st != FA_OK) return st;
    to_f32_kernel<<<16, 256>>>(s->aout_bf16, FA_DT_BF16, s->w_aout, (size_t)AD * M::D);
  }
  to_f32_kernel<<<1, 64>>>(aob, w->aout_b.dtype, s->b_aout, AD);
  FA_CUDA(h, cudaGetLastError());
  FA_CUDA(h, cudaDeviceSynchronize());
  s->weights = true;
  return FA_OK;
}

extern "C" fa_status fa_ma2_set_rope(fa_handle* h, const float* cos_tab, const float* sin_tab) {
  if (!h || !cos_tab || !sin_tab) return fail(h, FA_ERR_INVALID, "null argument");
  if (h->kind != FA_MODEL_MOLMOACT2 || !h->ma2) return fail(h, FA_ERR_INVALID, "not a MolmoAct2 handle");
  FA_CUDA(h, cudaSetDevice(h->device));
  const size_t n = (size_t)h->cfg.horizon * 48 * sizeof(float);
  FA_CUDA(h, cudaMemcpy(h->ma2->rope_cos, cos_tab, n, cudaMemcpyDefault));
  FA_CUDA(h, cudaMemcpy(h->ma2->rope_sin, sin_tab, n, cudaMemcpyDefault));
  return FA_OK;
}

fa_status ma2_set_modulation(fa_handle* h, const float* mods, const float* mod_final) {
  Ma2State* s = h->ma2;
  FA_CUDA(h, cudaSetDevice(h->device));
  const int S = h->cfg.num_steps, L = h->cfg.num_layers;
  FA_CUDA(h, cudaMemcpy(s->mods, mods, (size_t)S * L * 9 * M::D * 4, cudaMemcpyDefault));
  FA_CUDA(h, cudaMemcpy(s->mod_final, mod_final, (size_t)S * 2 * M::D * 4, cudaMemcpyDefault));
  s->mods_set = true;
  return FA_OK;
}

// Work plan: cross-attention units (observation, head, 128-key context chunk) in contiguous
// runs on the first CTAs; each GEMM matrix's units spread one per CTA before any CTA takes a
// second, ties broken by the CTA's total weight bytes.
static fa_status ma2_plan(fa_handle* h) {
  Ma2State* s = h->ma2;
  const int nblk = h->num_sms;
  // Cross-attention units per (observation, head, 128-key context chunk), merged per (token, head)
  // afterwards. Self-attention units take 8 query tokens, or all of an observation's tokens once the
  // (observation, head) pairs alone give half the SMs a unit (keys normalised once per unit:
  // 32 observations 22.3 -> 17.0 ms per chunk).
  {
    const char* q = getenv("FA_MA2_SELFQ");
    s->self_q = q ? (atoi(q) >= 32 ? 32 : 8) : (2 * s->B * M::H >= nblk ? 32 : 8);
  }
  // Whole units (every chunk of one (observation, head), online softmax, no merge stage) once the
  // (observation, head) pairs give a quarter of the SMs a unit (B200, context 493: 32 observations
  // 92.3 -> 74.6 ms per chunk, 8 observations 54.2 -> 48.5 ms; 1 observation 29.5 -> 31.0 ms, so
  // small batches keep the per-chunk units).
  {
    const char* w = getenv("FA_MA2_XWHOLE");
    s->cross_whole = w ? atoi(w) != 0 : 4 * s->B * M::H >= nblk;
  }
  std::vector<AttnUnit> au;
  for (int b = 0; b < s->B; ++b) {
    const int nch = (s->ctx[b] + M::KC - 1) / M::KC;
    for (int hh = 0; hh < M::H; ++hh) {
      if (s->cross_whole) {
        au.push_back({(uint16_t)b, (uint16_t)hh, fa::kWholeChunk, 0});
        continue;
      }
      for (int c = 0; c < nch; ++c) au.push_back({(uint16_t)b, (uint16_t)hh, (uint16_t)c, 0});
    }
  }
  std::vector<CtaPlan> plans(nblk);
  std::vector<long> load(nblk, 0);
  const int na = (int)au.size(), acta = std::min(na, nblk);
  for (int i = 0; i < nblk; ++i) {
    const int lo = i < acta ? (int)((long)na * i / acta) : 0, hi = i < acta ? (int)((long)na * (i + 1) / acta) : 0;
    plans[i].a_off = lo;
    plans[i].a_cnt = hi - lo;
    load[i] = 0;
    for (int k = lo; k < hi; ++k)  // a chunk's worth of work per unit, or every chunk of a whole unit
      load[i] += 8L * (au[k].chunk == fa::kWholeChunk ? (s->ctx[au[k].b] + M::KC - 1) / M::KC : 1);
  }
  std::vector<std::vector<GemmUnit>> per((size_t)nblk * M::NUM_MATS);
  const int order[M::NUM_MATS] = {M::MAT_GU, M::MAT_QKV, M::MAT_DN, M::MAT_SO, M::MAT_CQ, M::MAT_CO};
  // weight atoms per ring slot: 64 KB boxes for one token tile, 32 KB otherwise; divides every unit
  s->wg = s->NTILE == 64 ? fa::kMaxWG : 2;
  if (const char* e = getenv("FA_WG")) s->wg = std::max(1, std::min(s->wg, atoi(e)));
  // K-splits: the configured factor, stepped down to a smaller divisor of the K range while the
  // stage would hold more than two units per CTA (large batches fill the GPU through their
  // token groups instead)
  for (int m = 0; m < M::NUM_MATS; ++m) {
    int sp = s->split[m];
    const int katoms = kMatK[m] / 64, mtiles = kMatRows[m] / 128;
    while (sp > 1 && mtiles * sp * s->ngroups > 2 * nblk) {
      int d = sp - 1;
      while (d > 1 && katoms % d != 0) --d;
      sp = d;
    }
    s->split_eff[m] = sp;
  }
  for (int m = 0; m < M::NUM_MATS; ++m)
    while ((kMatK[m] / 64 / s->split_eff[m]) % s->wg != 0) s->wg >>= 1;
  // activation TMA box (32 KB) in K atoms, never more than divides every unit's K range
  s->ba = s->NTILE == 64 ? 4 : 2;
  for (int m = 0; m < M::NUM_MATS; ++m)
    while ((kMatK[m] / 64 / s->split_eff[m]) % s->ba != 0) s->ba >>= 1;
  // Token-major GEMMs (opt-in, FA_MA2_TM=1) while the bound batch is one tile of <= 64 tokens and
  // every unit's K range is whole 256-K chunks: activation chunks in three 32 KB staging slots,
  // 32 KB weight slots. Measured on B200 at C3 (bs=1): 33.5 ms per chunk against 29.3 ms for the
  // weight-major GEMMs (gate/up 1.73 -> 1.56 ms, but the single-chunk self-out / cross-q /
  // cross-out units and the down projection slower), so it is not the default here.
  {
    const char* e = getenv("FA_MA2_TM");
    bool tm = e && atoi(e) != 0 && s->NTILE == 64 && s->ngroups == 1;
    for (int m = 0; m < M::NUM_MATS; ++m) tm = tm && (kMatK[m] / 64 / s->split_eff[m]) % fa::kTmChunkAtoms == 0;
    s->tm = tm;
    if (tm) { s->wg = 2; s->ba = fa::kTmChunkAtoms; }
  }
  for (int oi = 0; oi < M::NUM_MATS; ++oi) {
    const int m = order[oi];
    const int mtiles = kMatRows[m] / 128, katoms = kMatK[m] / 64, split = s->split_eff[m], per_split = katoms / split;
    std::vector<int> cnt(nblk, 0);
    for (int g = 0; g < s->ngroups; ++g)
      for (int mt = 0; mt < mtiles; ++mt)
        for (int sp = 0; sp < split; ++sp) {
          int best = 0;
          for (int i = 1; i < nblk; ++i)
            if (cnt[i] < cnt[best] || (cnt[i] == cnt[best] && load[i] < load[best])) best = i;
          per[(size_t)best * M::NUM_MATS + m].push_back(
              {(uint16_t)mt, (uint16_t)(sp * per_split), (uint16_t)per_split, (uint16_t)sp, (uint16_t)g});
          cnt[best]++;
          load[best] += per_split * std::min(s->TG, s->NPAD / s->NTILE - g * s->TG);
        }
  }
  std::vector<GemmUnit> gu;
  const int tile = s->NTILE * 128;
  for (int i = 0; i < nblk; ++i) {
    int bb = tile, ng = 0;
    const int ntg = std::min(s->TG, s->NPAD / s->NTILE);  // token tiles per group
    for (int m = 0; m < M::NUM_MATS; ++m) {
      ng += (int)per[(size_t)i * M::NUM_MATS + m].size();
      for (const GemmUnit& x : per[(size_t)i * M::NUM_MATS + m]) bb = std::max(bb, (int)x.natoms * ntg * tile);
    }
    if (ng > fa::kMaxGU || plans[i].a_cnt > fa::kMaxAU)
      return fail(h, FA_ERR_INVALID, "batch too large for the per-CTA work lists (%d GEMM, %d attention units)", ng,
                  plans[i].a_cnt);
    bb = std::min(bb, std::min(fa::kMaxBBytes, fa::kMaxBAtoms * tile));
    bb = std::max(bb, tile * ntg * std::max(s->ba, s->wg));  // one activation box and weight slot per token tile
    if (plans[i].a_cnt > 0) bb = std::max(tile, std::min(bb, 64 * 1024));
    if (s->tm) bb = 3 * (int)fa::kTmChunkBytes;  // K = 768: three chunks per unit at most load at once
    plans[i].b_bytes = bb;
    const int work = std::max(bb, M::kMinWork) + fa::kStageBytes;
    plans[i].ring_slots = std::min(fa::kMaxRing, (fa::kSmemUse - work) / (s->wg * fa::kAtomBytes));
    if (plans[i].ring_slots < (s->tm ? 2 : 1))  // a token-major chunk of a 128-row unit takes 2 ring slots
      return fail(h, FA_ERR_INVALID, "shared-memory plan leaves no weight ring");
    for (int m = 0; m < M::NUM_MATS; ++m) {
      plans[i].g_off[m] = (int)gu.size();
      plans[i].g_cnt[m] = (int)per[(size_t)i * M::NUM_MATS + m].size();
      gu.insert(gu.end(), per[(size_t)i * M::NUM_MATS + m].begin(), per[(size_t)i * M::NUM_MATS + m].end());
    }
  }
  if (gu.size() > s->gcap) {
    if (s->d_gunits) cudaFree(s->d_gunits);
    FA_CUDA(h, cudaMalloc(&s->d_gunits, gu.size() * sizeof(GemmUnit)));
    s->gcap = gu.size();
  }
  if (au.size() > s->acap) {
    if (s->d_aunits) cudaFree(s->d_aunits);
    FA_CUDA(h, cudaMalloc(&s->d_aunits, std::max<size_t>(au.size(), 1) * sizeof(AttnUnit)));
    s->acap = au.size();
  }
  FA_CUDA(h, cudaMemcpy(s->d_gunits, gu.data(), gu.size() * sizeof(GemmUnit), cudaMemcpyHostToDevice));
  if (!au.empty()) FA_CUDA(h, cudaMemcpy(s->d_aunits, au.data(), au.size() * sizeof(AttnUnit), cudaMemcpyHostToDevice));
  FA_CUDA(h, cudaMemcpy(s->d_plans, plans.data(), plans.size() * sizeof(CtaPlan), cudaMemcpyHostToDevice));
  return FA_OK;
}

static fa_status ma2_params(fa_handle* h) {
  Ma2State* s = h->ma2;
  M::Params& p = s->params;
  memset(&p, 0, sizeof(p));
  const int L = h->cfg.num_layers;
  fa_status st;
  for (int m = 0; m < M::NUM_MATS; ++m)
    if ((st = make_map3(h, &p.maps[M::MAP_W_QKV + m], s->w[m], kMatK[m], (uint64_t)L * kMatRows[m], 128, s->wg)) != FA_OK)
      return st;
  const uint32_t ba = (uint32_t)s->ba;
  if ((st = make_map3(h, &p.maps[M::MAP_XN], s->xn, M::D, s->NPAD, s->NTILE, ba)) != FA_OK) return st;
  if ((st = make_map3(h, &p.maps[M::MAP_SATTN], s->sattn, M::D, s->NPAD, s->NTILE, ba)) != FA_OK) return st;
  if ((st = make_map3(h, &p.maps[M::MAP_CATTN], s->cattn, M::D, s->NPAD, s->NTILE, ba)) != FA_OK) return st;
  if ((st = make_map3(h, &p.maps[M::MAP_H], s->hbuf, M::F, s->NPAD, s->NTILE, ba)) != FA_OK) return st;
  // cross-attention context: K rows [B*L*LKPAD][768], 64 x 128 boxes at any 8-aligned dim offset
  // (a head starts at 96 h); V^T [B*L*768][LKPAD], boxes of 96 dims x 2 atoms of 64 keys
  if ((st = make_map2(h, &p.maps[M::MAP_KCTX], s->kctx, M::D, (uint64_t)s->B * L * s->LKPAD, 64, 128)) != FA_OK) return st;
  if ((st = make_map3(h, &p.maps[M::MAP_VTCTX], s->vctx, s->LKPAD, (uint64_t)s->B * L * M::D, 96, 2)) != FA_OK) return st;
  p.box_atoms = (int)ba;
  p.wg = s->wg;
  p.L = L; p.T = h->cfg.horizon; p.B = s->B; p.NT = s->NT; p.NPAD = s->NPAD; p.NTILE = s->NTILE; p.TG = s->TG;
  p.ngroups = s->ngroups; p.nsteps = h->cfg.num_steps; p.AD = h->cfg.action_dim; p.adim = s->adim; p.LKPAD = s->LKPAD;
  for (int m = 0; m < M::NUM_MATS; ++m) p.split[m] = s->split_eff[m];
  for (int m = 0; m < M::NUM_MATS; ++m) p.tg[m] = s->TG;
  p.self_q = s->self_q;
  {
    const char* e = getenv("FA_MA2_SELF_TC");  // 0: CUDA-core self-attention
    p.self_tc = !(e && atoi(e) == 0);
    p.cross_whole = s->cross_whole;
  }
  p.dt = 1.0f / (float)h->cfg.num_steps;
  p.invT = 1.0f / (float)h->cfg.horizon;
  p.gunits = s->d_gunits; p.aunits = s->d_aunits; p.plans = s->d_plans; p.ctx_len = s->d_ctx;
  p.mods = s->mods; p.mod_final = s->mod_final; p.rope_cos = s->rope_cos; p.rope_sin = s->rope_sin;
  for (int m = 0; m < M::NUM_MATS; ++m) p.bias[m] = s->bias[m];
  for (int m = 0; m < M::NUM_MATS; ++m) {
    p.wraw[m] = reinterpret_cast<const uint8_t*>(s->w[m]);
    p.wrow_bytes[m] = kMatK[m] * 2;
  }
  p.b_up = s->b_up;
  p.w_ain = s->w_ain; p.b_ain = s->b_ain; p.w_aout = s->w_aout; p.b_aout = s->b_aout;
  p.kctx = s->kctx; p.vctx = s->vctx;
  p.x_t = s->x_t; p.x = s->x; p.part = s->part; p.xn = s->xn; p.qkv = s->qkv; p.sattn = s->sattn;
  p.cattn = s->cattn; p.hbuf = s->hbuf; p.opart = s->opart; p.oml = s->oml;
  p.bar = h->ctrl; p.err = reinterpret_cast<int*>(h->ctrl + 1);
  ma2_set_debug(h);
  return FA_OK;
}

void ma2_set_debug(fa_handle* h) {
  if (!h || !h->ma2) return;
  M::Params& p = h->ma2->params;
  p.inject_barrier = h->params.inject_barrier;
  p.spin_limit = h->params.spin_limit ? h->params.spin_limit : (1u << 24);
  p.l2_ahead = l2_ahead_layers();
  p.trace = h->trace;
  p.trace_step = h->trace_step;
  p.trace_layer = h->trace_layer;
}

fa_status ma2_bind(fa_handle* h, int batch, const void* k, const void* v, int src_rows, const int* ctx_len,
                   cudaStream_t stream, const int* rowmap) {
  Ma2State* s = h->ma2;
  if (batch < 1 || batch > h->cfg.max_batch) return fail(h, FA_ERR_INVALID, "batch %d outside 1..%d", batch, h->cfg.max_batch);
  if (!ctx_len || !k || !v) return fail(h, FA_ERR_INVALID, "null argument");
  for (int b = 0; b < batch; ++b)
    if (ctx_len[b] < 1 || ctx_len[b] > src_rows || ctx_len[b] > h->cfg.max_prefix)
      return fail(h, FA_ERR_INVALID, "context length[%d]=%d outside 1..min(src_rows=%d, max_prefix=%d)", b, ctx_len[b],
                  src_rows, h->cfg.max_prefix);
  if (!is_device_ptr(k) || !is_device_ptr(v)) return fail(h, FA_ERR_INVALID, "k/v must be device pointers");
  FA_CUDA(h, cudaSetDevice(h->device));
  if (s->bound && !rowmap && batch == s->B && (int)s->ctx.size() == batch &&
      std::equal(ctx_len, ctx_len + batch, s->ctx.begin())) {
    // Same batch and context lengths: plan and parameters stay; the context is re-copied
    // asynchronously on `stream` (ordered after earlier launches on that stream).
    const int L_ = h->cfg.num_layers;
    const dim3 grid(std::max(1, s->LKPAD * M::D / 8 / 256 / 4), L_, batch);
    ma2_bind_ctx_kernel<<<grid, 256, 0, stream>>>((const bf16*)k, src_rows, s->d_ctx, nullptr, L_, s->LKPAD, s->kctx);
    ma2_bind_vt_kernel<<<dim3(s->LKPAD / 32, M::D / 32, batch * L_), dim3(32, 8), 0, stream>>>(
        (const bf16*)v, src_rows, s->d_ctx, nullptr, L_, s->LKPAD, s->vctx);
    FA_CUDA(h, cudaGetLastError());
    return FA_OK;
  }
  FA_CUDA(h, cudaStreamSynchronize(stream));
  const int T = h->cfg.horizon, L = h->cfg.num_layers;
  s->B = batch;
  s->NT = batch * T;
  s->NTILE = s->NT <= 64 ? 64 : 128;
  s->NPAD = round_up(s->NT, s->NTILE);
  s->TG = 256 / s->NTILE;
  s->ngroups = (s->NPAD / s->NTILE + s->TG - 1) / s->TG;
  s->LKPAD = round_up(h->cfg.max_prefix, M::KC);
  s->ctx.assign(ctx_len, ctx_len + batch);
  FA_CUDA(h, cudaMemcpy(s->d_ctx, ctx_len, batch * sizeof(int), cudaMemcpyHostToDevice));
  fa_status st;
  if ((st = ma2_plan(h)) != FA_OK) return st;
  if ((st = ma2_params(h)) != FA_OK) return st;
  const dim3 grid(std::max(1, s->LKPAD * M::D / 8 / 256 / 4), L, batch);
  ma2_bind_ctx_kernel<<<grid, 256, 0, stream>>>((const bf16*)k, src_rows, s->d_ctx, rowmap, L, s->LKPAD, s->kctx);
  ma2_bind_vt_kernel<<<dim3(s->LKPAD / 32, M::D / 32, batch * L), dim3(32, 8), 0, stream>>>(
      (const bf16*)v, src_rows, s->d_ctx, rowmap, L, s->LKPAD, s->vctx);
  FA_CUDA(h, cudaGetLastError());
  FA_CUDA(h, cudaStreamSynchronize(stream));
  s->bound = true;
  return FA_OK;
}

fa_status ma2_sample(fa_handle* h, int batch, const float* noise, float* out, cudaStream_t stream) {
  Ma2State* s = h->ma2;
  if (!s->weights) return fail(h, FA_ERR_STATE, "weights not loaded");
  if (!s->mods_set) return fail(h, FA_ERR_STATE, "modulations not set (fa_set_modulation)");
  if (!s->bound) return fail(h, FA_ERR_STATE, "context not bound");
  if (batch != s->B) return fail(h, FA_ERR_INVALID, "batch %d differs from the bound batch %d", batch, s->B);
  FA_CUDA(h, cudaSetDevice(h->device));
  const size_t bytes = (size_t)s->NT * h->cfg.action_dim * sizeof(float);
  M::Params& p = s->params;
  ma2_set_debug(h);
  p.stage_ns = h->timing ? h->stage_ns : nullptr;
  FA_CUDA(h, cudaMemsetAsync(h->ctrl, 0, fa::kCtrlWords * sizeof(unsigned int), stream));
  if (h->timing) FA_CUDA(h, cudaMemsetAsync(h->stage_ns, 0, fa::kMaxStages * sizeof(unsigned long long), stream));
  FA_CUDA(h, cudaMemcpyAsync(s->x_t, noise, bytes, cudaMemcpyDefault, stream));
  void* args[] = {&p};
  FA_CUDA(h, cudaLaunchCooperativeKernel(s->tm ? (const void*)M::ma2_denoise_kernel_tm : (const void*)M::ma2_denoise_kernel,
                                         dim3(h->num_sms), dim3(fa::kThreads), args,
                                         fa::kSmemDyn, stream));
  FA_CUDA(h, cudaMemcpyAsync(out, s->x_t, bytes, cudaMemcpyDefault, stream));
  h->last_launches = 1;
  h->last_stream = stream;
  return FA_OK;
}
