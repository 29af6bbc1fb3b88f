// On-device weight quantisers behind fa_quantize_fp8_rows / fa_quantize_nvfp4: they produce the
// codes and scales fa_pi05_load_weights_q takes, from bf16 / fp16 / fp32 weights already on the
// device (the reference quantises on the host inside HybridPi05._pack_weights,
// src/pi05/hybrid_model.py:105-110).
//
// Both follow the formulas stated in include/flashact.h operation by operation in fp32 (IEEE
// division, round-to-nearest-even conversions), so the codes are bit-identical to the same
// formulas evaluated with torch on the host.
#include "host_common.cuh"

namespace {

__device__ __forceinline__ unsigned char to_e4m3(float v) {
  return (unsigned char)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ float block_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();  // red is reused by consecutive rows
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float m = red[0];
  for (int i = 1; i < nw; ++i) m = fmaxf(m, red[i]);
  return m;
}

// FP8 per output row: scale = max(amax, 1e-8) / 448, code = E4M3(clamp(w / scale, -448, 448)).
__global__ void quant_fp8_rows_kernel(const void* w, int dt, size_t nrows, int K, unsigned char* codes, float* scale) {
  __shared__ float red[32];
  for (size_t r = blockIdx.x; r < nrows; r += gridDim.x) {
    const size_t base = r * (size_t)K;
    float m = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(load_as_float(w, base + k, dt)));
    const float s = fmaxf(block_max(m, red), 1e-8f) / 448.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const float q = fminf(fmaxf(load_as_float(w, base + k, dt) / s, -448.0f), 448.0f);
      codes[base + k] = to_e4m3(q);
    }
    if (threadIdx.x == 0) scale[r] = s;
  }
}

// NVFP4 pass 1: amax of each layer matrix, as float bits in tensor_scale[l] (zeroed by the
// host; non-negative floats order like their bit patterns).
__global__ void quant_amax_kernel(const void* w, int dt, size_t per_layer, float* tensor_scale) {
  __shared__ float red[32];
  const int l = blockIdx.y;
  float m = 0.f;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < per_layer; i += (size_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(load_as_float(w, (size_t)l * per_layer + i, dt)));
  m = block_max(m, red);
  if (threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned int*>(tensor_scale) + l, __float_as_uint(m));
}

// NVFP4 pass 2: tensor scale = max(amax / (448 * 6), 1e-12).
__global__ void quant_tscale_kernel(float* tensor_scale, int L) {
  const int l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l < L) tensor_scale[l] = fmaxf(tensor_scale[l] / 2688.0f, 1e-12f);
}

// Nearest E2M1 magnitude code of m in [0, 6]; on an exact tie the even code (mantissa bit 0).
// Candidates ascend, so a strict '<' keeps the lower index and the tie rule only has to prefer
// the upper one when that is the even code.
__device__ __forceinline__ int e2m1_nearest(float m) {
  const float vals[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  int best = 0;
  float bd = fabsf(m);
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    const float d = fabsf(m - vals[i]);
    if (d < bd || (d == bd && (i & 1) == 0)) { bd = d; best = i; }
  }
  return best;
}

// NVFP4 pass 3, one thread per 16-element block: block scale = E4M3(min(block amax / 6 / ts,
// 448)); x = w / (block scale * ts) (divided by 1 where that product is 0); code = sign |
// nearest E2M1 of min(|x|, 6), negative zero kept as code 0; even k in the low nibble.
__global__ void quant_nvfp4_kernel(const void* w, int dt, size_t nblocks, size_t blocks_per_layer,
                                   const float* tensor_scale, unsigned char* packed, unsigned char* bscale) {
  for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += (size_t)gridDim.x * blockDim.x) {
    const float ts = tensor_scale[b / blocks_per_layer];
    float v[16];
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = load_as_float(w, b * 16 + i, dt);
      m = fmaxf(m, fabsf(v[i]));
    }
    const unsigned char bs = to_e4m3(fminf(m / 6.0f / ts, 448.0f));
    __nv_fp8_e4m3 f;
    f.__x = bs;
    const float sc = (float)f * ts;
    const float div = sc > 0.f ? sc : 1.0f;
    uint2 out = make_uint2(0u, 0u);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float x = v[i] / div;
      const int idx = e2m1_nearest(fminf(fabsf(x), 6.0f));
      const unsigned code = (unsigned)idx | ((x < 0.f && idx > 0) ? 8u : 0u);
      if (i < 8) out.x |= code << (4 * i);
      else out.y |= code << (4 * (i - 8));
    }
    *reinterpret_cast<uint2*>(packed + b * 8) = out;
    bscale[b] = bs;
  }
}

int grid_for(size_t work, int per_block) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t want = (work + per_block - 1) / per_block;
  return (int)std::min<size_t>(want, (size_t)sms * 8);
}

fa_status check_args(const void* w, fa_dtype dt, int L, int rows, int K, std::initializer_list<const void*> outs) {
  if (!w) return fail(nullptr, FA_ERR_INVALID, "null weight pointer");
  if (dt != FA_DT_F32 && dt != FA_DT_BF16 && dt != FA_DT_F16) return fail(nullptr, FA_ERR_INVALID, "unsupported dtype %d", (int)dt);
  if (L < 1 || rows < 1 || K < 1) return fail(nullptr, FA_ERR_INVALID, "empty shape L=%d rows=%d K=%d", L, rows, K);
  if (!is_device_ptr(w)) return fail(nullptr, FA_ERR_INVALID, "the weights must be in device memory");
  for (const void* o : outs)
    if (!o || !is_device_ptr(o)) return fail(nullptr, FA_ERR_INVALID, "every output must be a device pointer");
  return FA_OK;
}

}  // namespace

extern "C" fa_status fa_quantize_fp8_rows(const void* w, fa_dtype dtype, int L, int rows, int K, unsigned char* codes,
                                          float* scale, fa_stream stream) {
  fa_status st = check_args(w, dtype, L, rows, K, {codes, scale});
  if (st != FA_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t nrows = (size_t)L * rows;
  quant_fp8_rows_kernel<<<grid_for(nrows, 1), 256, 0, s>>>(w, (int)dtype, nrows, K, codes, scale);
  FA_CUDA(nullptr, cudaGetLastError());
  return FA_OK;
}

extern "C" fa_status fa_quantize_nvfp4(const void* w, fa_dtype dtype, int L, int rows, int K, unsigned char* packed,
                                       unsigned char* block_scale, float* tensor_scale, fa_stream stream) {
  fa_status st = check_args(w, dtype, L, rows, K, {packed, block_scale, tensor_scale});
  if (st != FA_OK) return st;
  if (K % 16) return fail(nullptr, FA_ERR_INVALID, "K=%d is not a multiple of 16", K);
  if (reinterpret_cast<uintptr_t>(packed) % 8) return fail(nullptr, FA_ERR_INVALID, "packed must be 8-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t per_layer = (size_t)rows * K;
  FA_CUDA(nullptr, cudaMemsetAsync(tensor_scale, 0, (size_t)L * sizeof(float), s));
  const dim3 ag(std::max(1, grid_for(per_layer, 256 * 16) / std::max(1, L / 8 + 1)), L);
  quant_amax_kernel<<<ag, 256, 0, s>>>(w, (int)dtype, per_layer, tensor_scale);
  FA_CUDA(nullptr, cudaGetLastError());
  quant_tscale_kernel<<<(L + 127) / 128, 128, 0, s>>>(tensor_scale, L);
  FA_CUDA(nullptr, cudaGetLastError());
  const size_t nblocks = (size_t)L * rows * (K / 16);
  quant_nvfp4_kernel<<<grid_for(nblocks, 256), 256, 0, s>>>(w, (int)dtype, nblocks, per_layer / 16, tensor_scale,
                                                            packed, block_scale);
  FA_CUDA(nullptr, cudaGetLastError());
  return FA_OK;
}
