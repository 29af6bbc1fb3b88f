/*
 * flashact.h — C ABI of the B200 (sm_100a) flow-matching action-expert denoise engine.
 *
 * The reference (GautamSharda/FlashAct) exposes its denoise loop as one pybind11 function per
 * model, `launch(...)`, that takes pre-packed torch tensors plus caller-owned scratch:
 *   - pi0.5:     src/pi05/binding.cpp:28-68      (kernel src/pi05/mk6.cu:112)
 *   - MolmoAct2: src/molmoact2/binding.cpp:28-83 (kernel src/molmoact2/mk_ma2.cu:103)
 * Its three implicit steps — weight packing (src/pi05/hybrid_model.py:76-133), prefix-KV bind
 * (src/pi05/pack_weights.py:60-70 + hybrid_model.py:202-208) and sample = launch + x_t readback
 * (hybrid_model.py:215-222) — are explicit entry points here. Everything takes plain pointers and
 * sizes; no torch types cross this boundary. Every function returns a status and never throws.
 *
 * Threading: one handle belongs to one device. Calls on different handles may run concurrently
 * from different host threads; calls on one handle must be serialised by the caller.
 */
#ifndef FLASHACT_H_
#define FLASHACT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

typedef struct fa_handle fa_handle;
typedef struct CUstream_st* fa_stream; /* a cudaStream_t; NULL = legacy default stream */

typedef enum {
  FA_OK = 0,
  FA_ERR_INVALID = 1,     /* bad argument: shape, pointer, dtype, batch > capacity ...          */
  FA_ERR_CUDA = 2,        /* a CUDA runtime call failed (message in fa_last_error)             */
  FA_ERR_TIMEOUT = 3,     /* a bounded in-kernel wait (grid barrier, mbarrier) ran out          */
  FA_ERR_STATE = 4,       /* call order: sample before weights / KV were bound                  */
  FA_ERR_UNSUPPORTED = 5, /* feature or device not supported (e.g. not an sm_100 GPU)           */
  FA_ERR_OOM = 6
} fa_status;

typedef enum { FA_MODEL_PI05 = 0, FA_MODEL_MOLMOACT2 = 1 } fa_model_kind;
typedef enum { FA_WFMT_BF16 = 0, FA_WFMT_FP8 = 1, FA_WFMT_NVFP4 = 2 } fa_wfmt;
typedef enum { FA_DT_F32 = 0, FA_DT_BF16 = 1, FA_DT_F16 = 2 } fa_dtype;

/* Prefix-KV source layouts accepted by fa_bind_prefix_kv.
 * COMPACT_SPLIT_HALF: K and V as [B][L][src_rows][256], RoPE already applied to K in the
 *   split-half convention (pairs d, d+128), rows 0..valid_len-1 valid. This is the layout
 *   `compact_kv` produces (src/pi05/pack_weights.py:60-70).
 * FLASHRT_INTERLEAVED: same shape, but K's rotary pairs are interleaved (2d, 2d+1), as in the
 *   FlashRT encoder cache the reference ingests in its prologue (src/pi05/mk6.cu:258-277). */
typedef enum { FA_KV_COMPACT_SPLIT_HALF = 0, FA_KV_FLASHRT_INTERLEAVED = 1 } fa_kv_layout;

/* Model geometry. pi0.5: width 1024, 8 query heads, 1 KV head, head_dim 256, mlp 4096 are
 * fixed by the architecture; num_layers (18), horizon (50), action_dim (32), max_prefix,
 * max_batch and num_steps (10) are free. MolmoAct2: width 768, 8 heads, 8 KV heads (cross
 * attention), head_dim 96, mlp 3072 are fixed; num_layers (36), horizon (<= 32, 30 as wired in
 * the reference), action_dim (32), valid_action_dim (6 for SO100), max_prefix (the bound
 * cross-attention context, 493 tokens in the reference run), num_steps (10; t = 0 -> 1,
 * dt = +1/N). */
typedef struct fa_config {
  int num_layers;
  int width;
  int num_heads;
  int num_kv_heads;
  int head_dim;
  int mlp_dim;
  int horizon;    /* action tokens per observation (T)                  */
  int action_dim; /* AD                                                 */
  int max_prefix; /* capacity of the bound prefix KV per observation     */
  int max_batch;  /* observations per fa_sample_actions call             */
  int num_steps;  /* Euler steps N; pi0.5 integrates t = 1 -> 0, dt=-1/N */
  int valid_action_dim; /* MolmoAct2: action dims updated by the Euler step (the rest keep
                           their input value, src/molmoact2/mk_ma2.cu:565); 0 = all          */
} fa_config;

/* One weight tensor. ptr may be host or device memory (CUDA unified addressing decides). */
typedef struct fa_tensor {
  const void* ptr;
  fa_dtype dtype;
} fa_tensor;

/* pi0.5 action-expert weights, each stacked over layers where it is per layer, in the
 * [out][in] row-major layout of torch.nn.Linear. Names mirror the openpi keys the reference
 * reads in src/pi05/hybrid_model.py:94-133:
 *   layers.{i}.self_attn.{q,k,v,o}_proj.weight, mlp.{gate,up,down}_proj.weight,
 *   input_layernorm.dense.{weight,bias}, post_attention_layernorm.dense.{weight,bias},
 *   model.norm.dense.{weight,bias}, time_mlp_{in,out}.{weight,bias},
 *   action_{in,out}_proj.{weight,bias}. */
typedef struct fa_pi05_weights {
  fa_tensor wq, wk, wv, wo;         /* [L][2048][1024], [L][256][1024] x2, [L][1024][2048] */
  fa_tensor w_gate, w_up, w_down;   /* [L][4096][1024] x2, [L][1024][4096]                 */
  fa_tensor ln_in_w, ln_in_b;       /* [L][3072][1024], [L][3072]                          */
  fa_tensor ln_post_w, ln_post_b;   /* [L][3072][1024], [L][3072]                          */
  fa_tensor norm_w, norm_b;         /* [3072][1024], [3072]                                */
  fa_tensor time_in_w, time_in_b;   /* [1024][1024], [1024]                                */
  fa_tensor time_out_w, time_out_b; /* [1024][1024], [1024]                                */
  fa_tensor ain_w, ain_b;           /* [1024][AD], [1024]                                  */
  fa_tensor aout_w, aout_b;         /* [AD][1024], [AD]                                    */
} fa_pi05_weights;

/* Scales of one quantised GEMM weight (fa_pi05_load_weights_q).
 *  FP8 (E4M3, the reference's per-output-row scheme, src/pi05/hybrid_model.py:105-110): the
 *    weight's ptr holds uint8 codes [L][rows][K]; scale = fp32 [L][rows]; value = code * scale.
 *  NVFP4: ptr holds E2M1 codes, two per byte (even k in the low nibble) [L][rows][K/2];
 *    scale = E4M3 block scales [L][rows][K/16] (one per 16 consecutive k); tensor = fp32 [L];
 *    value = code * block_scale * tensor[l].
 * ptrs may be host or device memory. */
typedef struct fa_qscale {
  const void* scale;
  const float* tensor; /* NVFP4 only */
} fa_qscale;
typedef struct fa_pi05_qscales {
  fa_qscale wq, wk, wv, wo, w_gate, w_up, w_down;
} fa_pi05_qscales;

/* On-device quantisation of GEMM weights into the codes fa_pi05_load_weights_q takes (the
 * reference quantises on the host: FP8 branch of HybridPi05._pack_weights,
 * src/pi05/hybrid_model.py:105-110). w: device [L][rows][K] in `dtype`; outputs are device
 * memory; asynchronous on `stream`; bit-identical to the formulas below evaluated in fp32.
 *  FP8: scale[l][r] = max(amax_k |w|, 1e-8) / 448; codes[l][r][k] = E4M3(clamp(w / scale,
 *    -448, 448)), round to nearest even.
 *  NVFP4 (K % 16 == 0, packed 8-byte aligned): tensor_scale[l] = max(amax_{r,k} |w| / 2688,
 *    1e-12); block_scale[l][r][k/16] = E4M3(min(block amax / 6 / tensor_scale, 448));
 *    x = w / (block_scale * tensor_scale) (/ 1 where that is 0); code = nearest E2M1 of
 *    min(|x|, 6) (ties to the even code) with the sign of x (no negative zero); packed[l][r][k/2]
 *    holds even k in the low nibble.
 * Errors are read with fa_last_error(NULL). */
FA_API fa_status fa_quantize_fp8_rows(const void* w, fa_dtype dtype, int L, int rows, int K, unsigned char* codes,
                                      float* scale, fa_stream stream);
FA_API fa_status fa_quantize_nvfp4(const void* w, fa_dtype dtype, int L, int rows, int K, unsigned char* packed,
                                   unsigned char* block_scale, float* tensor_scale, fa_stream stream);

/* MolmoAct2 action-expert weights (benchmarks/molmoact2/eval_numerics.py:77-100 names), stacked
 * over the L blocks, [out][in] row-major: self_attn.qkv, self_attn.out_proj, cross_attn.q_proj,
 * cross_attn.out_proj, mlp.{gate,up,down}_proj (+ biases), action_embed, final_layer.linear. */
typedef struct fa_ma2_weights {
  fa_tensor w_qkv, b_qkv;     /* [L][2304][768], [L][2304] */
  fa_tensor w_so, b_so;       /* [L][768][768],  [L][768]  */
  fa_tensor w_cq, b_cq;       /* [L][768][768],  [L][768]  */
  fa_tensor w_co, b_co;       /* [L][768][768],  [L][768]  */
  fa_tensor w_gate, b_gate;   /* [L][3072][768], [L][3072] */
  fa_tensor w_up, b_up;       /* [L][3072][768], [L][3072] */
  fa_tensor w_down, b_down;   /* [L][768][3072], [L][768]  */
  fa_tensor ain_w, ain_b;     /* [768][AD], [768]          */
  fa_tensor aout_w, aout_b;   /* [AD][768], [AD] (aout used in bf16 like the reference) */
} fa_ma2_weights;

/* Creates a handle on `device`. Fails with FA_ERR_UNSUPPORTED on a GPU that is not sm_100. */
FA_API fa_status fa_create(fa_model_kind kind, const fa_config* cfg, int device, fa_handle** out);

/* Packs the weights into the engine's streaming layout on the device and computes, on the
 * device, the time embedding -> conditioning MLP -> per-layer adaRMS modulations for the
 * configured fixed schedule (reference: host-side in src/pi05/hybrid_model.py:111-128).
 * The ten conditioning tensors (ln_*, norm_*, time_*) may all be null: the modulations are then
 * set with fa_set_modulation, as the reference's launch() receives them precomputed
 * (src/pi05/binding.cpp:31). Synchronous. Replaces HybridPi05._pack_weights. */
FA_API fa_status fa_pi05_load_weights(fa_handle* h, const fa_pi05_weights* w, fa_wfmt fmt);

/* Quantised pi0.5 GEMM weights (fmt FA_WFMT_FP8 or FA_WFMT_NVFP4; see fa_qscale): the seven
 * GEMM tensors of `w` carry the codes (their dtype field is ignored), `s` their scales; the other
 * fields as for fa_pi05_load_weights. FP8: the codes are packed as they are and the FP8 kernel
 * streams them (half the bytes of bf16): each E4M3 tile is expanded exactly to bf16 in tensor
 * memory, where the MMAs read it as their A operand, and the row scale multiplies the fp32 accumulator, the
 * reference's W8A16 scheme (src/pi05/mk6.cu:90-94,204-205,219-220); codes must be 16-byte
 * aligned. (Environment FA_FP8_STREAM=0 at load time dequantises them into the bf16 layout
 * instead.) NVFP4: dequantised once on the device into the bf16 layout (value = code x block
 * scale x tensor scale, exact), so the model runs the bf16 kernel with the NVFP4 numerics.
 * Replaces the FP8 branch of HybridPi05._pack_weights. */
FA_API fa_status fa_pi05_load_weights_q(fa_handle* h, const fa_pi05_weights* w, fa_wfmt fmt, const fa_pi05_qscales* s);

/* MolmoAct2: packs the weights (bf16 GEMM weights, fp32 biases). Synchronous. The
 * modulations are an input of this model (the model's own modulation cache, which the reference
 * also passes to its kernel): set them with fa_set_modulation. */
FA_API fa_status fa_ma2_load_weights(fa_handle* h, const fa_ma2_weights* w);

/* MolmoAct2: RoPE tables of the self-attention, cos / sin [horizon][48] fp32 (host or device),
 * as the model's rope cache provides them (eval_numerics.py:110-113). fa_create installs the
 * theta = 10000 tables at positions 0..horizon-1 by default. */
FA_API fa_status fa_ma2_set_rope(fa_handle* h, const float* cos_tab, const float* sin_tab);

/* Overrides the modulations with precomputed ones. pi0.5: mods [num_steps][L][2][3072] fp32
 * (input / post-attention adaRMS; each scale|shift|gate) and mod_final [num_steps][3072]
 * (scale|shift used). MolmoAct2: mods [num_steps][L][3][3][768] ((self, cross, mlp) x (scale,
 * shift, gate)) and mod_final [num_steps][2][768] (scale, shift), src/molmoact2/binding.cpp:
 * 37-38. Device or host pointers. This is the form the reference's launch() receives
 * (src/pi05/binding.cpp:31, `mods`, `mod_final`). */
FA_API fa_status fa_set_modulation(fa_handle* h, const float* mods, const float* mod_final);

/* MolmoAct2: `k`, `v` are the per-block projected cross-attention context K and V,
 * [batch][L][src_rows][768] bf16 (8 heads x 96, K already normed as the model's prepare_context
 * produces it), with the first valid_len[b] rows valid (compacted); `layout` is ignored.
 * pi0.5: */
/* Binds the cached VLM prefix KV of `batch` observations (device pointers, bf16). K and V are
 * [batch][L][src_rows][256]; valid_len (host array, batch entries) gives each observation's
 * number of valid (compacted) prefix tokens, <= src_rows <= max_prefix. The action tokens'
 * RoPE positions start at valid_len (src/pi05/pack_weights.py:54-58). The copy / transpose /
 * de-interleave runs on `stream`. Replaces compact_kv + the kcache/vtcache fill.
 * A bind that changes the batch or any valid length re-plans the work and synchronises `stream`;
 * a rebind with the same batch and valid lengths (both models, unmasked) only re-copies the cache,
 * asynchronously on `stream` with no host synchronisation, like the reference's KV handoff inside
 * its launch (src/pi05/mk6.cu:258-277): issue it on the stream of the launches that read the cache. */
FA_API fa_status fa_bind_prefix_kv(fa_handle* h, int batch, const void* k, const void* v, int src_rows,
                            const int* valid_len, fa_kv_layout layout, fa_stream stream);

/* Same as fa_bind_prefix_kv for an UNcompacted prefix / context: keep is a device array
 * [batch][src_rows] (nonzero = valid token, e.g. the prefix pad mask, or MolmoAct2's
 * cross-attention mask == its max); the valid rows of each observation, in order, are gathered
 * on the device as the bound prefix (the compaction the reference does with torch ops before
 * its launch: compact_kv in src/pi05/pack_weights.py:60-70, and benchmarks/molmoact2/
 * eval_e2e.py:108-125). Synchronises `stream` once to read the valid counts back. */
FA_API fa_status fa_bind_prefix_kv_masked(fa_handle* h, int batch, const void* k, const void* v, int src_rows,
                                          const unsigned char* keep, fa_kv_layout layout, fa_stream stream);

/* Runs the whole N-step x L-layer Euler denoise loop as one cooperative megakernel.
 * noise: [batch][T][AD] fp32 initial x_1; actions_out: [batch][T][AD] fp32 final x_0. Either
 * may be host or device memory; host buffers are copied on `stream` inside the call. batch
 * must equal the batch of the last fa_bind_prefix_kv. Asynchronous w.r.t. the host when both
 * pointers are device (or pinned) memory; a barrier timeout is reported by the NEXT call that
 * synchronises (fa_sync) as FA_ERR_TIMEOUT. */
FA_API fa_status fa_sample_actions(fa_handle* h, int batch, const float* noise, float* actions_out,
                            fa_stream stream);

/* Waits for the handle's last launch and reports an in-kernel timeout / error flag. */
FA_API fa_status fa_sync(fa_handle* h, fa_stream stream);

/* Per-stage time of the last launch, in nanoseconds summed over the loop (block 0's view):
 * [0] embed/norm1 [1] qkv [2] attention [3] merge [4] o_proj [5] norm2 [6] gate/up [7] down
 * [8] final+euler. Enable with fa_set_stage_timing(h, 1) before sampling. n = array length.
 * A host `out` is filled synchronously; a device `out` is filled asynchronously on the stream of
 * the last fa_sample_actions (MolmoAct2 reports its 13 stages; entries past the model's count are 0). */
FA_API fa_status fa_set_stage_timing(fa_handle* h, int enable);
FA_API fa_status fa_get_stage_cycles(fa_handle* h, uint64_t* out, int n);

/* Number of kernel launches the last fa_sample_actions issued on the device (the megakernel
 * and any copies-by-kernel), for launch accounting. */
FA_API int fa_last_launch_count(fa_handle* h);

/* Test hook (host-side fault injection, no GPU fault): block 0 skips arriving at grid barrier
 * number `barrier_index` of the next launches (-1 = off) and every grid-barrier wait gives up
 * after `spin_limit` polls (0 = default). The launch then ends early with its error word set and
 * fa_sync reports FA_ERR_TIMEOUT; the context stays usable. Reset by fa_bind_prefix_kv. */
FA_API fa_status fa_set_fault_injection(fa_handle* h, int barrier_index, unsigned int spin_limit);

/* Diagnostics (builds compiled with -DFA_TRACE; otherwise FA_ERR_UNSUPPORTED): with step >= 0,
 * arm a trace of one (step, layer) of the following launches;
 * with step < 0, copy n stamps to host_out, laid out [9 stages][num_SMs][16]: per CTA the
 * stage-start clock64, then offsets in cycles (first weight tile ready, activation tiles ready,
 * last MMA committed, first accumulator ready, epilogue done, barrier arrive), the absolute
 * clock64 at which the producer issued the stage's first weight tile and the offset at which
 * the activation loads were issued. */
FA_API fa_status fa_debug_trace(fa_handle* h, int step, int layer, unsigned long long* host_out, int n);

/* Allocation-free variant of the conditioning step of fa_pi05_load_weights; it has no
 * counterpart in the reference. For callers that cannot allocate device memory at the point
 * where they need the modulations (a control process whose memory budget is fixed after start-up,
 * a host that hands out memory only from its own pool). It computes the time embedding ->
 * conditioning MLP -> adaRMS modulations for the fixed schedule t_s = 1 - s/num_steps, writing
 * mods_out [num_steps][num_layers][2][3072] and mod_final_out [num_steps][3072] (device fp32,
 * the layout fa_set_modulation takes) on `stream`, asynchronously. Only the conditioning fields of
 * `w` are read (ln_*, norm_*, time_*), and they must already be in device memory.
 * Scratch: a static 600 KB device array inside the library (at most 50 steps), held by every GPU
 * that loads the library until exit; the call allocates nothing itself. Under CUDA's lazy module
 * loading, the library's device module (and with it that array) is loaded on a device the first
 * time the library touches it there, and that load takes device memory: make the first call on
 * each device at start-up, before the memory budget is fixed and before any stream capture. Every
 * call looks the array up (cudaGetSymbolAddress) on the current device, so it keeps working after
 * a cudaDeviceReset. Weights and outputs must be memory of the current device (or managed).
 * A CUDA error already pending on the thread is reported (FA_ERR_CUDA) and left in place; nothing
 * is launched then. All calls share the array: calls that overlap on the GPU race. The last error
 * message is read with fa_last_error(NULL). Rejects num_steps > 50. */
FA_API fa_status fa_pi05_modulations_noalloc(const fa_pi05_weights* w, int num_layers, int num_steps,
                                             float* mods_out, float* mod_final_out, fa_stream stream);

/* Last error message of the handle (or of the thread's last failed fa_create when h is NULL). */
FA_API const char* fa_last_error(fa_handle* h);

FA_API void fa_destroy(fa_handle* h);

#ifdef __cplusplus
}
#endif
#endif /* FLASHACT_H_ */
