// Types and constants shared by host and device code of every denoise megakernel in this
// library (pi0.5 and MolmoAct2): the per-CTA work plan, shared-memory budget, trace slots and
// in-kernel error codes.
#pragma once
#include <cstdint>

namespace fa {

constexpr int kThreads = 192;              // warp 0 producer, warp 1 MMA, warps 2-5 epilogue / vector work
constexpr int kAtomBytes = 128 * 64 * 2;   // one 128-row x 64-col bf16 atom, 128-byte swizzle
constexpr int kSmemUse = 224 * 1024;       // dynamic shared memory used (ring + work area)
constexpr int kSmemDyn = kSmemUse + 1024;  // + alignment slack
// Weight atoms per ring slot (Params::wg, 1..kMaxWG): one 3D TMA box of wg consecutive K-atoms
// of a 128-row tile. A single SM sustains about 4 TMA loads in flight, so larger boxes raise its
// streaming rate (measured on B200: 16 KB boxes ~68 GB/s per SM; 64 KB boxes ~120 GB/s with two
// in flight).
constexpr int kMaxWG = 4;
constexpr int kMaxRing = 12;               // weight-ring slots
// FP8 weight streaming (pi0.5): the ring holds E4M3 tiles (half the bytes); the epilogue warps
// expand each slot to bf16 straight into tensor memory, where the MMAs read their A operand
// (TMEM columns [kAColF8, 512): kASlotsF8 slots of kASlotColsF8 columns; accumulators in
// [0, 2 x kAccColsF8)).
constexpr int kAccColsF8 = 128;            // accumulator columns per buffer (token columns <= 128)
constexpr int kAColF8 = 256;               // first TMEM column of the A slots
constexpr int kASlotsF8 = 2;
constexpr int kASlotColsF8 = 128;          // 256 K-values of bf16 (2 per 32-bit column)
// Token-major GEMMs (one tile of <= 64 tokens): activation K-chunks of 4 atoms (256 K) staged in up
// to four 32 KB slots, read there by the MMAs; one accumulator of <= 128 columns at [0, 128).
constexpr int kTmChunkAtoms = 4;
constexpr uint32_t kTmChunkBytes = 64 * 128 * kTmChunkAtoms;
constexpr uint32_t kTmASlots = 3;  // A-slot barriers (FP8 expansion uses 2)
constexpr int kMaxBBytes = 128 * 1024;     // activation (B operand) area of a GEMM CTA, upper bound
constexpr int kMaxBAtoms = 16;             // activation atoms resident at once
constexpr int kMaxGU = 48;                 // GEMM units per CTA per layer (all matrices)
constexpr int kMaxAU = 48;                 // attention units per CTA per layer
constexpr int kMaxMats = 6;                // GEMM matrices per layer
constexpr int kStageBytes = 16 * 1024;     // epilogue staging area
constexpr int kMaxStages = 16;             // traced stage kinds
constexpr int kCtrlWords = 2;  // launch control words, zeroed before each launch: grid-barrier counter, error word

struct GemmUnit {
  uint16_t mtile;   // 128-row tile of the packed weight
  uint16_t katom0;  // first 64-wide K atom
  uint16_t natoms;  // K atoms in this unit
  uint16_t split;   // index of the fp32 partial slice it writes (K-split stages)
  uint16_t grp;     // token group: token tiles [grp * TG, grp * TG + TG) (one TMEM accumulator)
  uint16_t half;    // 0: all 128 rows of the tile; 1 / 2: rows [0, 64) / [64, 128) only (the
                    // weight stream of one SM halves; the MMA stays M = 128, rows 64..127 of its
                    // result are ignored)
};
struct AttnUnit {
  uint16_t b, hp, chunk, is_suffix;  // observation, head (pair), key chunk, action-token chunk flag
};
constexpr uint16_t kWholeChunk = 0xFFFF;  // AttnUnit::chunk of a unit that covers every key chunk
struct CtaPlan {
  int g_off[kMaxMats], g_cnt[kMaxMats];  // GEMM units of this CTA per matrix, same for every layer
  int a_off, a_cnt;                      // attention units of this CTA
  int ring_slots;                        // weight-ring depth
  int b_bytes;                           // activation area of this CTA
};

enum TraceSlot : int {
  kTrStart = 0,      // absolute clock64 at stage start (after the barrier); others are offsets
  kTrMmaW0 = 1,      // MMA lane: first weight atom ready / attention: Q and K ready
  kTrMmaB0 = 2,      // MMA lane: activation atoms ready / attention: V ready
  kTrMmaDone = 3,    // MMA lane: last accumulator committed
  kTrEpiAcc0 = 4,    // epilogue: first accumulator ready
  kTrEpiDone = 5,    // epilogue: stage work done
  kTrBarArrive = 6,  // barrier thread: arrived
  kTrProdIssue = 7,  // producer: ABSOLUTE clock64 when it issued this stage's first weight atom
  kTrMmaPre = 8,     // MMA lane: activation loads issued
  kTrStride = 16
};

// Error codes written to the launch's error word.
enum KernelError : int { KERR_BARRIER = 1, KERR_PRODUCER = 2, KERR_MMA = 3, KERR_EPI = 4, KERR_ATTN = 5, KERR_CONV = 6 };

}  // namespace fa
