// Host-side pieces shared by the model engines behind the C ABI: the handle, error reporting,
// device allocation, weight staging / row-gather packing, and TMA descriptor builders.
#pragma once
#include <cudaTypedefs.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/flashact.h"
#include "fa_pi05.cuh"

using bf16 = __nv_bfloat16;
using fa::pi05::Params;
using fa::GemmUnit;
using fa::AttnUnit;
using fa::CtaPlan;

struct Ma2State;

// ------------------------------------------------------------------ handle
struct fa_handle {
  fa_model_kind kind;
  fa_config cfg;
  int device = 0;
  int num_sms = 0;
  std::string err;
  bool weights_ready = false, kv_ready = false, timing = false;
  int last_launches = 0;
  cudaStream_t last_stream = nullptr;  // stream of the last fa_sample_actions
  int split_o = 8, split_dn = 8, attn_penalty = 8;
  int split_o_eff = 4, split_dn_eff = 8;  // K-splits used for the bound batch
  int bmax_bytes = 64 * 1024;  // activation-area cap of a GEMM CTA
  int ring_max = 12;           // weight-ring depth cap
  int wg = 4;                  // weight atoms per ring slot (bound batch)
  bool half_units = true;      // 64-row QKV / gate-up units at one token tile
  // FP8 weight streaming (pi0.5 weights loaded as FP8 codes): E4M3 codes and per-row scales of
  // QKV, O, gate/up, down in the packed row order; the FP8 kernel streams them
  bool fp8_stream = false;
  bool tm = false;
  bool attn_whole = false;     // pi0.5: whole-unit attention (two-pass softmax, no merge)             // token-major GEMM kernel (bound batch = one tile of <= 64 tokens)
  unsigned char* w8[4] = {nullptr, nullptr, nullptr, nullptr};
  float* ws8[4] = {nullptr, nullptr, nullptr, nullptr};
  // bound batch
  int B = 0, NT = 0, NPAD = 0, NTILE = 64, TG = 4, ngroups = 1, LPAD = 0;
  int tgm[4] = {4, 4, 4, 4};  // pi0.5: token tiles per group of each GEMM matrix (QKV, O, gate/up, down)
  std::vector<int> valid_len;
  // device memory
  std::vector<void*> allocs;
  bf16 *w_qkv = nullptr, *w_o = nullptr, *w_gu = nullptr, *w_dn = nullptr;
  float *mods = nullptr, *mod_final = nullptr;
  float *w_ain = nullptr, *b_ain = nullptr, *w_aout = nullptr, *b_aout = nullptr;
  float *x_t = nullptr, *x = nullptr, *part = nullptr, *oml = nullptr;
  bf16* opart = nullptr;
  bf16 *xn = nullptr, *attn = nullptr, *hbuf = nullptr, *q = nullptr, *sk = nullptr, *svt = nullptr;
  bf16 *kcache = nullptr, *vtcache = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  int *d_valid = nullptr, *d_nchunks = nullptr;
  unsigned int* ctrl = nullptr;  // [0] barrier counter, [1] error word
  int* d_rowmap = nullptr;       // masked binds: [batch][src_rows] source row of each kept row
  int* d_counts = nullptr;       // masked binds: kept rows per observation
  size_t rowmap_cap = 0;
  unsigned long long* stage_ns = nullptr;
  GemmUnit* d_gunits = nullptr;
  AttnUnit* d_aunits = nullptr;
  CtaPlan* d_plans = nullptr;
  size_t n_gunits_cap = 0, n_aunits_cap = 0;
  unsigned long long* trace = nullptr;
  int trace_step = -1, trace_layer = -1;
  Params params;
  Ma2State* ma2 = nullptr;  // MolmoAct2 engine state (FA_MODEL_MOLMOACT2 handles)
};

extern thread_local std::string g_create_err;

static inline fa_status fail(fa_handle* h, fa_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (h) h->err = buf; else g_create_err = buf;
  return st;
}
#define FA_CUDA(h, call)                                                                        \
  do {                                                                                          \
    cudaError_t e_ = (call);                                                                    \
    if (e_ != cudaSuccess) return fail(h, FA_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                       __FILE__, __LINE__);                                     \
  } while (0)

template <class T>
static inline fa_status dalloc(fa_handle* h, T** out, size_t count) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, count * sizeof(T) + 16);
  if (e != cudaSuccess) return fail(h, FA_ERR_OOM, "cudaMalloc(%zu bytes): %s", count * sizeof(T), cudaGetErrorString(e));
  e = cudaMemset(p, 0, count * sizeof(T) + 16);
  if (e != cudaSuccess) return fail(h, FA_ERR_CUDA, "cudaMemset: %s", cudaGetErrorString(e));
  h->allocs.push_back(p);
  *out = reinterpret_cast<T*>(p);
  return FA_OK;
}

// Masked binds: for each observation b (one block each), the source rows whose keep flag is set,
// in order: rowmap[b][i] = i-th kept row, counts[b] = number kept (the reference's
// compact_kv / `kv[0][mask]` gather, src/pi05/pack_weights.py:60-70,
// benchmarks/molmoact2/eval_e2e.py:108-125, done on the device).
static __global__ void rowmap_kernel(const unsigned char* keep, int src_rows, int* rowmap, int* counts) {
  __shared__ int warp_tot[32];
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, w = t >> 5, nt = blockDim.x;
  const int per = (src_rows + nt - 1) / nt, r0 = t * per, r1 = min(src_rows, r0 + per);
  const unsigned char* kb = keep + (size_t)b * src_rows;
  int mine = 0;
  for (int r = r0; r < r1; ++r) mine += kb[r] != 0;
  int incl = mine;  // inclusive scan over the block
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[w] = incl;
  __syncthreads();
  if (w == 0) {
    int v = lane < nt / 32 ? warp_tot[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    warp_tot[lane] = v;  // inclusive prefix of warp totals
  }
  __syncthreads();
  int pos = incl - mine + (w > 0 ? warp_tot[w - 1] : 0);
  for (int r = r0; r < r1; ++r)
    if (kb[r]) rowmap[(size_t)b * src_rows + pos++] = r;
  if (t == nt - 1) counts[b] = pos;
}


// Builds the row map of a masked bind on `stream` (into the handle's reusable buffers) and
// returns the kept-row counts on the host (the bind plans its attention work from them).
static inline fa_status masked_rows(fa_handle* h, int batch, int src_rows, const unsigned char* keep, cudaStream_t stream,
                             std::vector<int>& counts) {
  if (!keep || batch < 1 || src_rows < 1) return fail(h, FA_ERR_INVALID, "masked bind: bad mask arguments");
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, keep) != cudaSuccess || a.type != cudaMemoryTypeDevice) {
    cudaGetLastError();
    return fail(h, FA_ERR_INVALID, "masked bind: the keep mask must be device memory");
  }
  const size_t need = (size_t)batch * src_rows;
  if (need > h->rowmap_cap) {
    int *rm = nullptr, *ct = nullptr;
    if (cudaMalloc(&rm, need * sizeof(int)) != cudaSuccess) return fail(h, FA_ERR_OOM, "masked bind: row map");
    if (cudaMalloc(&ct, (size_t)batch * sizeof(int) + 16) != cudaSuccess) {
      cudaFree(rm);
      return fail(h, FA_ERR_OOM, "masked bind: counts");
    }
    h->allocs.push_back(rm);
    h->allocs.push_back(ct);
    h->d_rowmap = rm;
    h->d_counts = ct;
    h->rowmap_cap = need;
  }
  rowmap_kernel<<<batch, 1024, 0, stream>>>(keep, src_rows, h->d_rowmap, h->d_counts);
  FA_CUDA(h, cudaGetLastError());
  counts.resize(batch);
  FA_CUDA(h, cudaMemcpyAsync(counts.data(), h->d_counts, batch * sizeof(int), cudaMemcpyDeviceToHost, stream));
  FA_CUDA(h, cudaStreamSynchronize(stream));
  return FA_OK;
}

static inline bool is_device_ptr(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// Layers of weights the producer warps prefetch into L2 ahead of their loads (FA_L2_AHEAD, 0..4;
// default 0).
static inline int l2_ahead_layers() {
  const char* e = getenv("FA_L2_AHEAD");
  return e ? std::max(0, std::min(4, atoi(e))) : 0;
}

static size_t dtype_size(fa_dtype t) { return t == FA_DT_F32 ? 4 : 2; }

__device__ __forceinline__ float load_as_float(const void* p, size_t i, int dt) {
  if (dt == FA_DT_F32) return reinterpret_cast<const float*>(p)[i];
  if (dt == FA_DT_BF16) return __bfloat162float(reinterpret_cast<const bf16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// ------------------------------------------------------------------ device helper kernels
// Row-gather pack: dst[l][r][k] = bf16(src_{sel(r)}[l][row(r)][k]). rowmap[r] = (source id, row).
struct PackSrc {
  const void* ptr[3];
  int dtype[3];
  int rows[3];  // rows per layer of each source
  // quantised sources (fa_pi05_load_weights_q): 0 = plain dtype, 1 = FP8 E4M3 codes x per-row
  // fp32 scale, 2 = NVFP4 (E2M1 codes x E4M3 per-16 block scale x fp32 per-layer scale)
  int quant;
  const void* scale[3];
  const float* tensor[3];
};
// E2M1 (sign, 2 exponent bits with bias 1, 1 mantissa bit): 0, 0.5, 1, 1.5, 2, 3, 4, 6.
__device__ __forceinline__ float e2m1_value(unsigned v) {
  const unsigned e = (v >> 1) & 3u, m = v & 1u;
  const float mag = e == 0 ? 0.5f * (float)m : (1.0f + 0.5f * (float)m) * (float)(1u << (e - 1));
  return (v & 8u) ? -mag : mag;
}
__device__ __forceinline__ float e4m3_value(unsigned char c) {
  __nv_fp8_e4m3 f;
  f.__x = c;
  return (float)f;
}
static __global__ void pack_rows_kernel(PackSrc s, const int2* rowmap, bf16* dst, int R, int K, int L) {
  const size_t total = (size_t)L * R * K;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int k = (int)(i % K);
    const size_t lr = i / K;
    const int r = (int)(lr % R), l = (int)(lr / R);
    const int2 m = rowmap[r];
    const size_t srow = (size_t)l * s.rows[m.x] + m.y;
    const size_t si = srow * K + k;
    float v;
    if (s.quant == 1) {
      v = e4m3_value(reinterpret_cast<const unsigned char*>(s.ptr[m.x])[si]) *
          reinterpret_cast<const float*>(s.scale[m.x])[srow];
    } else if (s.quant == 2) {
      const unsigned char b = reinterpret_cast<const unsigned char*>(s.ptr[m.x])[si >> 1];
      const float bs = e4m3_value(reinterpret_cast<const unsigned char*>(s.scale[m.x])[srow * (K / 16) + k / 16]);
      v = e2m1_value((k & 1) ? (b >> 4) : (b & 15u)) * bs * s.tensor[m.x][l];
    } else {
      v = load_as_float(s.ptr[m.x], si, s.dtype[m.x]);
    }
    dst[i] = __float2bfloat16(v);
  }
}
// FP8 streaming pack: codes dst[l][r][:] = src_{sel(r)}[l][row(r)][:] (16-byte copies) and the
// row scales dscale[l][r] alongside.
static __global__ void pack_codes_kernel(PackSrc s, const int2* rowmap, unsigned char* dst, float* dscale, int R, int K,
                                         int L) {
  const int kv = K / 16;
  const size_t total = (size_t)L * R * kv;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int v = (int)(i % kv);
    const size_t lr = i / kv;
    const int r = (int)(lr % R), l = (int)(lr / R);
    const int2 m = rowmap[r];
    const size_t srow = (size_t)l * s.rows[m.x] + m.y;
    *reinterpret_cast<uint4*>(dst + lr * K + v * 16) =
        *reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned char*>(s.ptr[m.x]) + srow * K + v * 16);
    if (v == 0) dscale[lr] = reinterpret_cast<const float*>(s.scale[m.x])[srow];
  }
}
static __global__ void to_f32_kernel(const void* src, int dt, float* dst, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = load_as_float(src, i, dt);
}
static inline int round_up(int a, int b) { return (a + b - 1) / b * b; }

// ------------------------------------------------------------------ TMA descriptors
static inline PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}
// 3D bf16 map viewing a row-major [rows][K] array as [K/64 atoms][rows][64]: one box
// {64, box_rows, box_atoms} lands in shared memory as box_atoms consecutive 128B-swizzled atoms.
// 2D bf16 map over a row-major [rows][K] matrix: boxes of box_k x box_rows (box_k x 2 bytes = 128 for
// the 128-byte swizzle), at any K offset that is a multiple of 8 elements.
static inline fa_status make_map2(fa_handle* h, CUtensorMap* m, const void* base, uint64_t K, uint64_t rows,
                                  uint32_t box_k, uint32_t box_rows) {
  auto enc = get_encode();
  if (!enc) return fail(h, FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {K * 2};
  cuuint32_t box[2] = {box_k, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(h, FA_ERR_CUDA, "cuTensorMapEncodeTiled (2D) failed (%d)", (int)r);
  return FA_OK;
}

static inline fa_status make_map3(fa_handle* h, CUtensorMap* m, const void* base, uint64_t K, uint64_t rows,
                           uint32_t box_rows, uint32_t box_atoms) {
  auto enc = get_encode();
  if (!enc) return fail(h, FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {64, rows, K / 64};
  cuuint64_t strides[2] = {K * 2, 128};
  cuuint32_t box[3] = {64, box_rows, box_atoms};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(h, FA_ERR_CUDA, "cuTensorMapEncodeTiled (3D) failed (%d)", (int)r);
  return FA_OK;
}

// 3D E4M3 map viewing a row-major [rows][K] byte array as [K/128][rows][128]: one box
// {128, box_rows, box_n} lands as box_n consecutive 128B-swizzled boxes of box_rows x 128 bytes.
static inline fa_status make_map3_u8(fa_handle* h, CUtensorMap* m, const void* base, uint64_t K, uint64_t rows,
                              uint32_t box_rows, uint32_t box_n) {
  auto enc = get_encode();
  if (!enc) return fail(h, FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {128, rows, K / 128};
  cuuint64_t strides[2] = {K, 128};
  cuuint32_t box[3] = {128, box_rows, box_n};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(h, FA_ERR_CUDA, "cuTensorMapEncodeTiled (3D, u8) failed (%d)", (int)r);
  return FA_OK;
}

// Returns a device pointer holding `bytes` of `p` (staging host data into `tmp` when needed).
static inline fa_status stage_bytes(fa_handle* h, const void* p, size_t bytes, const char* name, const void** dptr,
                             std::vector<void*>& tmp) {
  if (!p) return fail(h, FA_ERR_INVALID, "'%s' is null", name);
  if (is_device_ptr(p)) { *dptr = p; return FA_OK; }
  void* d = nullptr;
  if (cudaMalloc(&d, bytes) != cudaSuccess) return fail(h, FA_ERR_OOM, "staging '%s' (%zu bytes)", name, bytes);
  tmp.push_back(d);
  FA_CUDA(h, cudaMemcpy(d, p, bytes, cudaMemcpyHostToDevice));
  *dptr = d;
  return FA_OK;
}

// Returns a device pointer holding `t` (staging host data into `tmp` when needed).
static inline fa_status stage_tensor(fa_handle* h, const fa_tensor& t, size_t count, const char* name, const void** dptr,
                              std::vector<void*>& tmp) {
  if (!t.ptr) return fail(h, FA_ERR_INVALID, "weight '%s' is null", name);
  if (t.dtype != FA_DT_F32 && t.dtype != FA_DT_BF16 && t.dtype != FA_DT_F16)
    return fail(h, FA_ERR_INVALID, "weight '%s' has unsupported dtype %d", name, (int)t.dtype);
  if (is_device_ptr(t.ptr)) { *dptr = t.ptr; return FA_OK; }
  void* d = nullptr;
  const size_t bytes = count * dtype_size(t.dtype);
  if (cudaMalloc(&d, bytes) != cudaSuccess) return fail(h, FA_ERR_OOM, "staging '%s' (%zu bytes)", name, bytes);
  tmp.push_back(d);
  FA_CUDA(h, cudaMemcpy(d, t.ptr, bytes, cudaMemcpyHostToDevice));
  *dptr = d;
  return FA_OK;
}

static inline fa_status pack_codes(fa_handle* h, const std::vector<int2>& rowmap, PackSrc src, unsigned char* dst, float* dscale,
                            int K, std::vector<void*>& tmp) {
  int2* d_map = nullptr;
  FA_CUDA(h, cudaMalloc(&d_map, rowmap.size() * sizeof(int2)));
  tmp.push_back(d_map);
  FA_CUDA(h, cudaMemcpy(d_map, rowmap.data(), rowmap.size() * sizeof(int2), cudaMemcpyHostToDevice));
  pack_codes_kernel<<<h->num_sms * 8, 256>>>(src, d_map, dst, dscale, (int)rowmap.size(), K, h->cfg.num_layers);
  FA_CUDA(h, cudaGetLastError());
  return FA_OK;
}

static inline fa_status pack_matrix(fa_handle* h, const std::vector<int2>& rowmap, PackSrc src, bf16* dst, int K,
                             std::vector<void*>& tmp) {
  int2* d_map = nullptr;
  FA_CUDA(h, cudaMalloc(&d_map, rowmap.size() * sizeof(int2)));
  tmp.push_back(d_map);
  FA_CUDA(h, cudaMemcpy(d_map, rowmap.data(), rowmap.size() * sizeof(int2), cudaMemcpyHostToDevice));
  pack_rows_kernel<<<h->num_sms * 8, 256>>>(src, d_map, dst, (int)rowmap.size(), K, h->cfg.num_layers);
  FA_CUDA(h, cudaGetLastError());
  return FA_OK;
}


// MolmoAct2 engine (host_ma2.cu), reached through the C ABI's model dispatch.
fa_status ma2_create(const fa_config& cfg, int device, fa_handle* h);
fa_status ma2_bind(fa_handle* h, int batch, const void* k, const void* v, int src_rows, const int* valid_len,
                   cudaStream_t s, const int* rowmap);
fa_status ma2_sample(fa_handle* h, int batch, const float* noise, float* out, cudaStream_t s);
fa_status ma2_set_modulation(fa_handle* h, const float* mods, const float* mod_final);
void ma2_set_debug(fa_handle* h);
void ma2_destroy(fa_handle* h);
