// step_kernel.cuh -- the persistent NCA step kernel for sm_100a.
//
// One CTA per SM.  Each step, every instance's cells are processed in tiles of 128 consecutive
// cells (global cell index g = inst * H * W + i * W + j).  Per tile:
//
//   loader warp    1-D bulk copies (cp.async.bulk) of the tile's halo window (cells
//                  g0-W-1 .. g0+128+W) of the previous state into a shared-memory stage laid out
//                  [chunk][cell][16 B], each chunk row ending in a padding cell
//   stencil warps  one thread per tile row and half of the channels: 3x3 perception (4 heads,
//                  head-major z[k*C + c] as nca.model.KernelPerception, src/nca/model.py:
//                  175-178; neighbours outside the board read the padding cell) written as bf16
//                  (bf16 hi + lo in split mode) into tensor memory, the A operand of GEMM1; the
//                  half-0 warps also write the per-row fire / given flags of the step
//   MMA thread     GEMM1 acc1 = z W1^T (tcgen05.mma kind::f16, A from TMEM, B = fc1.weight in
//                  128B-swizzled smem), then after the hidden epilogue GEMM2 acc2 = h W2^T
//   epilogue warps E1: h = relu(acc1 + b1) -> bf16 back into TMEM (A operand of GEMM2);
//                  E2: dx = acc2 + b2, fire mask (+ noise), x' = x + f*dx, clamp, store
//                  (src/nca/model.py:527-559, 430-438)
//   confidence     (confidence fire rules only) after the epilogue has stored a tile, read its
//   warps          readout slices back, evaluate the head and store each cell's fire
//                  probability of the next step (src/nca/model.py:566-593, 596-633)
//
// Resident form (StepCfg::RESIDENT): each CTA keeps groups of whole instances in shared memory
// for all steps of the launch (bf16 hi parts in two alternating buffers, the stencil's source,
// and lo parts), reading the state from HBM when a group starts and writing it at its last step.
//
// Tensor memory (512 columns x 128 lanes): NZ slots holding z and one accumulator region
// holding acc1, then h (bf16, over the columns already read) and acc2.  Every wait is bounded; a
// wait that runs out records NCA_ERR_TIMEOUT in the control words and the CTA drains and exits.
#pragma once
#include <cuda_bf16.h>

#include "ptx.cuh"

namespace nca {

constexpr int kTileM = 128;
// Warp roles: warp group 0 holds the MMA warp (0), the loader warp (1) and the two confidence
// warps (2, 3; idle without the confidence rules); warp groups 1-2 the 8 stencil warps (4..11);
// warp groups 3-4 the 8 epilogue warps (12..19).  With 20 warps a sub-partition hosts 5 of them,
// so every thread has 96 registers.
constexpr int kStencilWarp0 = 4;
constexpr int kEpiWarp0 = 12;

constexpr int pow2ceil(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

// Channels of one epilogue thread in E2 (two epilogue parts split the channels).
__host__ __device__ constexpr int epi_part_channels(int C) { return C / 2; }

// State layout of a model (see state_get): bf16 mode keeps hi + lo bf16 parts when C >= 64 (the
// MMA work per cell hides the extra packing, and a step moves 512 instead of 768 bytes per
// cell), else an fp32 master plus a bf16 mirror for the stencil; split mode keeps fp32.
__host__ __device__ constexpr bool hilo_layout(int C, bool bf16) { return bf16 && C >= 64; }

template <int C_, int HD_, bool SPLIT_, bool NOISE_ = false, bool TILEDEP_ = false,
          bool ADAPTIVE_ = false, bool RESIDENT_ = false>
struct StepCfg {
  static constexpr int C = C_;
  static constexpr bool NOISE = NOISE_;  // test-time state noise (a separate instantiation)
  // fire decisions on the cell's confidence (fire modes 2..5): the epilogue computes each cell's
  // fire probability for the next step from the values it stores, the stencil draws against it
  static constexpr bool ADAPTIVE = ADAPTIVE_;
  // Shared-memory-resident mode: each CTA takes groups of whole instances and keeps their state
  // in shared memory for all steps of the launch (bf16 hi parts in two buffers that alternate
  // between steps -- the stencil's source --, lo parts in place); no grid barrier, HBM is read
  // at a group's start and written at its last step.  bf16 mode below 64 channels.
  static constexpr bool RESIDENT = RESIDENT_;
  // steps ordered by per-tile step counters (StepArgs::tile_steps) instead of a grid barrier
  static constexpr bool TILEDEP = TILEDEP_;
  static constexpr int P = 4 * C_;
  static constexpr int HD = HD_;
  static constexpr bool SPLIT = SPLIT_;
  static constexpr bool SRC_BF16 = !SPLIT_;
  static constexpr bool HILO = hilo_layout(C_, !SPLIT_);
  static constexpr int SRC_BYTES = SRC_BF16 ? 2 : 4;
  static constexpr int ROWB = C * SRC_BYTES;         // bytes of one cell in a window stage
  static constexpr int NCH = ROWB / 16;              // 16-byte chunks per cell
  static constexpr int CPC = 16 / SRC_BYTES;         // channels per chunk
  static constexpr int ZPARTS = SPLIT ? 2 : 1;
  static constexpr int KMAX = P > HD ? P : HD;
  static constexpr int SLOT_COLS = ZPARTS * KMAX / 2;
  static constexpr int NZ = (2 * SLOT_COLS + HD <= 512) ? 2 : 1;
  static constexpr int ACC_COL = NZ * SLOT_COLS;
  // bf16 mode keeps h in the accumulator region (each epilogue thread overwrites the columns it
  // has read), so a z slot is free as soon as GEMM1 is done; acc2 then sits in columns
  // [HD/4, HD/2) of the region.  Split mode writes h (hi and lo) over the consumed z slot.
  static constexpr bool H_IN_ACC = !SPLIT_;
  // Accumulator regions (HD columns each, tile it uses region it % NACC).  Two fit beside the z
  // slots when HD <= 128: GEMM1 of the next tile then runs while the epilogue finishes this one.
  static constexpr int NACC = (H_IN_ACC && ACC_COL + 2 * HD <= 512) ? 2 : 1;
  static constexpr int TMEM_COLS = pow2ceil(ACC_COL + NACC * HD);
  static constexpr int ACC2_COL = ACC_COL + (H_IN_ACC ? HD / 4 : 0);
  static constexpr int W1_BYTES = HD * P * 2;
  static constexpr int W2_BYTES = C * HD * 2;
  // Epilogue warps per tensor-memory lane quarter ("parts"): 2, each with E1 of one GEMM1
  // N-half and E2 of half of the channels.  The code also runs with 4 parts (two per N-half,
  // the second writing h after the first has read its accumulator columns): measured slower at
  // 72 registers per thread, the limit of 28 warps.
  static constexpr int EPI_PARTS = 2;
  static_assert(C_ / EPI_PARTS == epi_part_channels(C_), "epilogue channel shares");
  static constexpr int PARTS_PER_HALF = EPI_PARTS / 2;
  static constexpr int EPI_WARPS = 4 * EPI_PARTS;
  static constexpr int CH = C_ / EPI_PARTS;             // channels of one epilogue thread in E2
  static constexpr int NUM_WARPS = kEpiWarp0 + EPI_WARPS;
  static constexpr int THREADS = NUM_WARPS * 32;
  static_assert(ACC_COL + NACC * HD <= 512, "tensor memory budget");
  static_assert(C % 16 == 0 && HD % 32 == 0 && HD <= 256 && P % 64 == 0 && HD % 64 == 0,
                "shape constraints of the UMMA tiles");
  static_assert(NCH % 2 == 0, "stencil channel halves");
  static_assert(!H_IN_ACC || C <= HD / 4, "acc2 must fit next to h in the accumulator region");
  static_assert(NUM_WARPS % 4 == 0 && CH % 8 == 0, "warp groups and E2 channel shares");
  static_assert(EPI_WARPS <= 8, "progress words (resident form, confidence warps)");
  static_assert(!RESIDENT || (!SPLIT && !HILO && !NOISE && !ADAPTIVE && !TILEDEP),
                "the resident mode is a bf16-mode kernel without noise or confidence rules");
};

// n / d for 0 <= n < 2^31 with a multiply-high and a shift (Granlund & Montgomery, "Division by
// invariant integers using multiplication", PLDI'94): q = (umulhi(n, m) + n) >> l with
// l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1.
struct FastDiv {
  unsigned m;
  int l;
};
__host__ __device__ __forceinline__ FastDiv make_fastdiv(unsigned d) {
  int l = 0;
  while ((1ull << l) < d) ++l;
  FastDiv f;
  f.m = (unsigned)((((1ull << 32) * ((1ull << l) - d)) / d) + 1);
  f.l = l;
  return f;
}
__device__ __forceinline__ unsigned fdiv(unsigned n, FastDiv f) { return (__umulhi(n, f.m) + n) >> f.l; }

struct StepArgs {
  int n_inst, H, W, HW, K;
  FastDiv div_hw, div_w, div_k;
  long long total, n_tiles, inst_offset;
  int n_steps;
  long long step0;
  int stages, win_cells;
  // resident mode: instances per group, cells per group (res_inst * HW), groups
  int res_inst;
  long long res_cells, n_groups;
  float pad[64];  // state of the cells outside a board (zero padding: 0), by channel
  int c_in, in_off, c_out, out_off, n_out, fixed_taps;
  float taps[4][9];
  float head_w[16][16];
  float head_b[16];
  const uint8_t* wimg;
  const uint8_t* wimg_lo;  // residual image (split mode with fp32 weights) or null
  int head_kind;
  const float* b1;
  const float* b2;
  const uint8_t* given;
  const float* clamp;
  const int* inst_row;
  const int* inst_id;
  float* master[2];
  uint16_t* mirror[2];
  int cur;
  int fire_mode;
  float p_fire, ad_scale, ad_bias, p_low, tau;
  int given_confident;
  unsigned long long seed;
  const uint8_t* masks;
  const float* uniforms;
  unsigned* updates;
  int noise_mode;
  float noise_p_t, noise_p_s, noise_sigma;
  long long noise_until;
  const float* noise;
  unsigned* tile_steps;  // per tile: steps of this launch whose stores are complete (TILEDEP)
  float* fire_p;         // per cell: fire probability of the next step (adaptive rules)
  int* ctrl;
  unsigned long long timeout_ns;
};

constexpr int kBarSlots = 48;  // mbarriers in the shared-memory layout
constexpr int kHeadFloats = 16 * 16 + 16;  // a copy of the readout head in shared memory
template <int N>
struct IntTag {
  static constexpr int value = N;
};

// Shared-memory layout (offsets from a 1024-byte aligned base).
template <class Cfg>
struct SmemLayout {
  int w1, w2, w1lo, w2lo, win, rlo, pwin, head, b1, b2, flags, bars, misc, total;
  __host__ __device__ SmemLayout(int stages, int win_cells, bool lo) {
    w1 = 0;
    w2 = w1 + Cfg::W1_BYTES;
    w1lo = w2 + Cfg::W2_BYTES;  // the residual image, when present, follows (same layout)
    w2lo = w1lo + Cfg::W1_BYTES;
    win = ((lo ? w2lo + Cfg::W2_BYTES : w1lo) + 1023) & ~1023;
    rlo = (win + stages * (win_cells + 1) * Cfg::ROWB + 15) & ~15;  // + the padding cell
    // resident mode: the window stages are the two buffers of the hi parts of the group's state
    // (win_cells = cells of a group) and the lo parts follow, [chunk][cell][16 B]
    pwin = rlo + (Cfg::RESIDENT ? win_cells * Cfg::ROWB : 0);
    // adaptive rules: the tile's fire probabilities, one fp32 per row, with each window stage,
    // and each confidence warp's copy of the head (16 x 16 weights, 16 biases)
    head = pwin + (Cfg::ADAPTIVE ? stages * kTileM * 4 : 0);
    b1 = head + (Cfg::ADAPTIVE ? 2 * kHeadFloats * 4 : 0);
    b2 = b1 + Cfg::HD * 4;
    flags = b2 + Cfg::C * 4;
    bars = (flags + 4 * kTileM + 7) & ~7;
    misc = bars + kBarSlots * 8;
    total = misc + 64;
  }
};

// The tiles of one CTA, as one or more passes.  Streaming: one pass, tiles t = blockIdx.x +
// k * grid of the whole batch at every step.  Resident: one pass per group of instances
// (groups blockIdx.x + k * grid), tiles 0 .. T - 1 of the group at every step.  The global cell
// of row m of tile t is cell0 + t * 128 + m; rows at or past `lim` are not cells.
struct Pass {
  long long t0, t1, dt, cell0, lim;
};
template <class Cfg>
__device__ __forceinline__ long long pass_count(const StepArgs& A, int grid) {
  if constexpr (Cfg::RESIDENT) return (A.n_groups - blockIdx.x + grid - 1) / grid;
  return 1;
}
template <class Cfg>
__device__ __forceinline__ Pass pass_of(const StepArgs& A, long long ps, int grid) {
  Pass P;
  if constexpr (Cfg::RESIDENT) {
    P.cell0 = (blockIdx.x + ps * grid) * A.res_cells;
    P.lim = P.cell0 + A.res_cells < A.total ? P.cell0 + A.res_cells : A.total;
    P.t0 = 0;
    P.t1 = (P.lim - P.cell0 + kTileM - 1) / kTileM;
    P.dt = 1;
  } else {
    P.cell0 = 0;
    P.lim = A.total;
    P.t0 = blockIdx.x;
    P.t1 = A.n_tiles;
    P.dt = grid;
  }
  return P;
}

constexpr int kMaxStages = 4;  // window stages
#ifndef NCA_TILEDEP_PER_CTA
#define NCA_TILEDEP_PER_CTA 8
#endif
// launches with at most this many tiles per CTA order their steps by per-tile step counters
constexpr int kTileDepPerCta = NCA_TILEDEP_PER_CTA;
enum BarId {
  BAR_WIN_FULL = 0,   // +stage (4)
  BAR_WIN_EMPTY = 4,  // +stage (4)
  BAR_Z_FULL = 8,     // +slot (2)
  BAR_Z_EMPTY = 10,   // +slot (2)
  // +accumulator region (2) each:
  BAR_ACC_FULL = 12,    // first half of GEMM1 (hidden units 0 .. HD/2)
  BAR_ACC_FULL_B = 14,  // second half of GEMM1 (hidden units HD/2 .. HD)
  BAR_H_FULL = 16,      // first half of the hidden epilogue
  BAR_H_FULL_B = 18,    // second half of the hidden epilogue
  BAR_ACC2_FULL = 20,   // GEMM2
  BAR_ACC_EMPTY = 22,   // acc2 read: the region is free
  BAR_WEIGHTS = 24,
  BAR_DRAIN = 25,
  BAR_FLAGS = 26,       // +ring index (4): per-row fire/given flags of a tile are written
  // +lane quarter + 4 * GEMM1 half (8): the first epilogue part of a half has read its
  // accumulator columns (bf16 mode, two parts per half: the second part writes h over them)
  BAR_PAIR = 30,
  BAR_RES_LOADED = 38,   // resident mode: the epilogue warps have loaded a group's state
  BAR_COUNT = 39
};
static_assert(BAR_COUNT <= kBarSlots, "barrier area of the shared-memory layout");

// Failure sites reported in ctrl[1].
enum Where {
  W_MMA_ZFULL = 1, W_MMA_ACCEMPTY, W_MMA_HFULL, W_MMA_WEIGHTS, W_LOAD_EMPTY, W_LOAD_GRID,
  W_ST_WINFULL, W_ST_ZEMPTY, W_E1_ACC, W_E2_ACC2, W_DRAIN, W_E2_FLAGS, W_PUBLISH, W_E1_PAIR, W_CONF, W_RES
};

// A window stage is laid out [chunk][window cell][16 B]: lanes that read the same chunk of
// consecutive cells touch consecutive 16-byte words (no bank conflicts), and every chunk of the
// window is a copy of contiguous rows of the tiled state layout (a few 1-D bulk copies).

// Warp-converged bounded wait (all 32 lanes call it).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const FailState& fs,
                                          int where) {
  const int lane = threadIdx.x & 31;
  uint64_t start = 0;
  if (lane == 0) start = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    bool done = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, done)) return true;
    int give_up = 0;
    if ((it & 63) == 63 && lane == 0) {
      if (should_abort(fs)) give_up = 1;
      else if (global_timer_ns() - start > fs.timeout_ns || it > (1u << 28)) {
        report_failure(fs, 4, where);
        give_up = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, give_up, 0)) return false;
    if (it > 128) __nanosleep(32);
  }
}

// Warp-converged bounded wait until each of the n progress words in shared memory is >= need
// (resident mode: the epilogue warps' count of finished tiles).
__device__ __forceinline__ bool wait_progress(const unsigned* words, int n, unsigned need,
                                              const FailState& fs, int where) {
  const int lane = threadIdx.x & 31;
  uint64_t start = 0;
  for (uint32_t it = 0;; ++it) {
    bool done = true;
    if (lane < n) {
      unsigned v;
      asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(words + lane)) : "memory");
      done = v >= need;
    }
    if (__all_sync(0xffffffffu, done)) return true;
    int give_up = 0;
    if (lane == 0 && (it & 63) == 63) {
      const uint64_t now = global_timer_ns();
      if (start == 0) start = now;
      if (should_abort(fs)) give_up = 1;
      else if (now - start > fs.timeout_ns || it > (1u << 28)) {
        report_failure(fs, 4, where);
        give_up = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, give_up, 0)) return false;
    __nanosleep(32);
  }
}

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) |   // LBO = 16 B (unused)
         ((uint64_t)(1024 >> 4) << 32) |                              // SBO = 1024 B
         ((uint64_t)1 << 46) |                                        // descriptor version
         ((uint64_t)2 << 61);                                         // SWIZZLE_128B
}

// The start-address field holds address >> 4 in the low 14 bits; shared memory is < 256 KB,
// so adding (bytes >> 4) moves the start address without touching the other fields.
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t bytes) {
  return d + (uint64_t)(bytes >> 4);
}

__device__ __forceinline__ uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------------------------------
// Stencil of one chunk: fixed identity / Sobel-x / Sobel-y / Laplacian taps.
//   Sobel-x = [[-1,0,1],[-2,0,2],[-1,0,1]] / 8 (src/nca/model.py:200), Sobel-y = its transpose,
//   Laplacian = [[1,2,1],[2,-12,2],[1,2,1]] / 16.
// Neighbours named by position:  a b c / d e f / g h k.
__device__ __forceinline__ void fixed_taps4(float a, float b, float c, float d, float e, float f,
                                            float g, float h, float k, float& sx, float& sy,
                                            float& lap) {
  float L = fmaf(2.f, d, a) + g;
  float R = fmaf(2.f, f, c) + k;
  float T = fmaf(2.f, b, a) + c;
  float B = fmaf(2.f, h, g) + k;
  sx = (R - L) * 0.125f;
  sy = (B - T) * 0.125f;
  float s = T + B;
  s = fmaf(2.f, d, s);
  s = fmaf(2.f, f, s);
  s = fmaf(-12.f, e, s);
  lap = s * 0.0625f;
}

// The state of a cell channel.  fp32 layout: master [tile][C/4][128][4] (split mode, and bf16
// mode below 64 channels, with a bf16 copy [tile][C/8][128][8] in `mirror` for the stencil).
// hi/lo layout (bf16 mode, C >= 64): two bf16 values [tile][C/8][128][8], hi = bf16(x) in
// `mirror` (the array the stencil reads) and lo = bf16(x - hi) in `master` (reinterpreted), so
// x = hi + lo carries about 16 significant bits and a step reads and writes 4 bytes per channel.
__host__ __device__ __forceinline__ long long sidx8(long long g, int C, int c) {
  return (((g >> 7) * (C / 8) + (c >> 3)) * 128 + (g & 127)) * 8 + (c & 7);
}
__host__ __device__ __forceinline__ long long sidx4(long long g, int C, int c) {
  return (((g >> 7) * (C / 4) + (c >> 2)) * 128 + (g & 127)) * 4 + (c & 3);
}
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
__device__ __forceinline__ float state_get(const float* master, const uint16_t* mirror, int C,
                                           long long g, int c) {
  if (mirror && hilo_layout(C, true)) {
    const long long i = sidx8(g, C, c);
    return bf16_bits_to_f32(mirror[i]) + bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(master)[i]);
  }
  return master[sidx4(g, C, c)];
}
__device__ __forceinline__ void state_put(float* master, uint16_t* mirror, int C, long long g, int c,
                                          float v) {
  if (mirror && hilo_layout(C, true)) {
    const long long i = sidx8(g, C, c);
    const uint16_t h = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    mirror[i] = h;
    reinterpret_cast<uint16_t*>(master)[i] = __bfloat16_as_ushort(__float2bfloat16_rn(v - bf16_bits_to_f32(h)));
  } else {
    master[sidx4(g, C, c)] = v;
    if (mirror) mirror[sidx8(g, C, c)] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  }
}

// Readout of one cell from its readout slice xs[0 .. c_out) (src/nca/model.py:596-633):
// kind 0 (head "mlp"): scores head_w x + head_b, confidence the max softmax;
// kind 1 (head "l2"): rows of head_w are the output-token embeddings e_o, score
// 1 / (1 + sqrt(|x - e_o|^2 + 1e-8)), confidence the best score.  arg is the first best token
// (torch.argmax).  head_w and head_b are zero outside n_out x c_out and xs is zero from c_out on
// (copy_head on the host, the callers' slices), so every row sums all 16 channels without a check
// per channel: the extra terms are exact zeros and leave each score as the sum over c < c_out in
// increasing order.  Only the rows o < n_out are evaluated.
// MAXC: a compile-time bound on c_out (the channels past c_out are zeros, see above); the callers
// on the hot path pick the smallest of 4, 9, 16 that holds c_out (head_readout_auto).
template <int MAXC = 16>
__device__ __forceinline__ void head_readout(int kind, int n_out, int c_out, const float (&hw)[16][16],
                                             const float (&hb)[16], const float (&xs)[16],
                                             float& conf, int& arg) {
  (void)c_out;
  float sc[16];
  float best = -3.402823466e38f;
  int a = 0;
#pragma unroll
  for (int o = 0; o < 16; ++o) {
    sc[o] = 0.f;
    if (o < n_out) {
      float v;
      if (kind == 1) {
        float d2 = 0.f;
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
          const float d = xs[c] - hw[o][c];
          d2 = fmaf(d, d, d2);
        }
        v = 1.f / (1.f + sqrtf(d2 + 1e-8f));
      } else {
        v = hb[o];
#pragma unroll
        for (int c = 0; c < MAXC; ++c) v = fmaf(hw[o][c], xs[c], v);
      }
      sc[o] = v;
      if (v > best || o == 0) { best = v; a = o; }
    }
  }
  arg = a;
  if (kind == 1) {
    conf = fminf(fmaxf(best, 0.f), 1.f);
    return;
  }
  float den = 0.f;
#pragma unroll
  for (int o = 0; o < 16; ++o)
    if (o < n_out) den += expf(sc[o] - best);
  conf = fminf(fmaxf(1.f / den, 0.f), 1.f);
}

__device__ __forceinline__ void head_readout_auto(int kind, int n_out, int c_out, const float (&hw)[16][16],
                                                  const float (&hb)[16], const float (&xs)[16],
                                                  float& conf, int& arg) {
  if (c_out <= 4) head_readout<4>(kind, n_out, c_out, hw, hb, xs, conf, arg);
  else if (c_out <= 9) head_readout<9>(kind, n_out, c_out, hw, hb, xs, conf, arg);
  else head_readout<16>(kind, n_out, c_out, hw, hb, xs, conf, arg);
}

// The head weights of a model as the kernels read them: head_w / head_b zero outside
// n_out x c_out (head_readout sums over all 16 channels of every row).
__host__ __forceinline__ void copy_head(float (&dw)[16][16], float (&db)[16], const float (&sw)[16][16],
                                        const float (&sb)[16], int n_out, int c_out) {
  for (int o = 0; o < 16; ++o) {
    db[o] = o < n_out ? sb[o] : 0.f;
    for (int c = 0; c < 16; ++c) dw[o][c] = (o < n_out && c < c_out) ? sw[o][c] : 0.f;
  }
}

// The fire probability of a cell under the confidence rules: fire modes 2 and 3 the continuous
// rule p = scale * (1 - conf) + bias, modes 4 and 5 the reference's threshold rule
// (src/nca/model.py:566-593): p_low for confident cells (conf > tau, or given cells when
// given_confident), else p_fire.
__device__ __forceinline__ float adaptive_prob(int mode, float conf, bool given, float scale, float bias,
                                               float p_low, float tau, float p_fire, int given_confident) {
  if (mode >= 4) return (conf > tau || (given && given_confident)) ? p_low : p_fire;
  return scale * (1.f - conf) + bias;
}

// The confidences of NR cells (head_readout's conf) for the confidence warps, mlp head: the
// weights come from this warp's copy in shared memory (hw [16][16], then hb [16]; broadcast
// loads shared by the cells) and two scores per packed f32x2 FMA, each accumulated like
// head_readout's (head_b first, then channels in increasing order, one rounding per fma), so
// the results are bit-identical to it.  MAXC / MAXO bound c_out / n_out at compile time: the
// code has no branch (scores past n_out are masked out of the max and the sum), so the
// compiler interleaves the independent FMA chains.
template <int MAXC, int MAXO, int NR>
__device__ __forceinline__ void head_confidence(int n_out, const float* s_head, const float (&x)[NR][MAXC],
                                                float (&conf)[NR]) {
  static_assert(MAXO % 2 == 0 && MAXO <= 16 && MAXC <= 16, "head bounds");
  float sc[NR][MAXO];
#pragma unroll
  for (int o = 0; o < MAXO; o += 2) {
    float2 v[NR];
    const float2 bias = *reinterpret_cast<const float2*>(s_head + 256 + o);
#pragma unroll
    for (int q = 0; q < NR; ++q) v[q] = bias;
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const float2 w = f2(s_head[o * 16 + c], s_head[(o + 1) * 16 + c]);
#pragma unroll
      for (int q = 0; q < NR; ++q) v[q] = __ffma2_rn(w, f2(x[q][c], x[q][c]), v[q]);
    }
#pragma unroll
    for (int q = 0; q < NR; ++q) {
      sc[q][o] = v[q].x;
      sc[q][o + 1] = v[q].y;
    }
  }
#pragma unroll
  for (int q = 0; q < NR; ++q) {
    float b = sc[q][0];
#pragma unroll
    for (int o = 1; o < MAXO; ++o) b = (o < n_out && sc[q][o] > b) ? sc[q][o] : b;
    float d = 0.f;
#pragma unroll
    for (int o = 0; o < MAXO; ++o) {
      const float e = expf(sc[q][o] - b);
      d += o < n_out ? e : 0.f;
    }
    conf[q] = fminf(fmaxf(1.f / d, 0.f), 1.f);
  }
}

// Row r of tile t of the state the epilogue stored at a step (buffer `out`): its readout slice,
// channels out_off .. out_off + c_out - 1 (c_out <= MAXC).  slice_issue loads the chunks that
// hold it (the hi/lo layout: bf16 hi and lo parts in 8-channel chunks, the value is hi + lo; the
// fp32 layout: float4 chunks) without using them, so their latency overlaps other work;
// slice_values converts them to xs[0 .. c_out), zeros after.  The loads are coherent: the
// epilogue wrote these values during this launch.
template <class Cfg, int MAXC>
struct SliceRaw {
  static constexpr int CW = Cfg::HILO ? 8 : 4;              // channels per chunk
  static constexpr int NK = (2 * (CW - 1) + MAXC) / CW;      // chunks a slice can span
  uint4 w[Cfg::HILO ? 2 * NK : NK];                          // hi chunks then lo chunks / float4 bits
};

template <class Cfg, int MAXC>
__device__ __forceinline__ void slice_issue(const StepArgs& A, int out, long long t, int r, SliceRaw<Cfg, MAXC>& R) {
  using S = SliceRaw<Cfg, MAXC>;
  constexpr int NCHUNK = Cfg::C / S::CW;
  const int k0 = A.out_off / S::CW, d = A.out_off - k0 * S::CW;
  const int nk = (d + A.c_out + S::CW - 1) / S::CW;
#pragma unroll
  for (int j = 0; j < S::NK; ++j) {
    const int k = k0 + j;
    const bool in = j < nk && k < NCHUNK;
    const long long idx = ((t * NCHUNK + (in ? k : 0)) << 7) + r;
    if constexpr (Cfg::HILO) {
      R.w[j] = in ? reinterpret_cast<const uint4*>(A.mirror[out])[idx] : make_uint4(0, 0, 0, 0);
      R.w[S::NK + j] = in ? reinterpret_cast<const uint4*>(A.master[out])[idx] : make_uint4(0, 0, 0, 0);
    } else {
      R.w[j] = in ? reinterpret_cast<const uint4*>(A.master[out])[idx] : make_uint4(0, 0, 0, 0);
    }
  }
}

template <class Cfg, int MAXC>
__device__ __forceinline__ void slice_values(const StepArgs& A, const SliceRaw<Cfg, MAXC>& R, float (&xs)[MAXC]) {
  using S = SliceRaw<Cfg, MAXC>;
  const int d = A.out_off % S::CW;
  float v[S::NK * S::CW];
#pragma unroll
  for (int j = 0; j < S::NK; ++j) {
    if constexpr (Cfg::HILO) {
      const uint32_t hh[4] = {R.w[j].x, R.w[j].y, R.w[j].z, R.w[j].w};
      const uint32_t ll[4] = {R.w[S::NK + j].x, R.w[S::NK + j].y, R.w[S::NK + j].z, R.w[S::NK + j].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[j * 8 + 2 * e] = bf16lo_to_f32(hh[e]) + bf16lo_to_f32(ll[e]);
        v[j * 8 + 2 * e + 1] = bf16hi_to_f32(hh[e]) + bf16hi_to_f32(ll[e]);
      }
    } else {
      v[j * 4] = __uint_as_float(R.w[j].x);
      v[j * 4 + 1] = __uint_as_float(R.w[j].y);
      v[j * 4 + 2] = __uint_as_float(R.w[j].z);
      v[j * 4 + 3] = __uint_as_float(R.w[j].w);
    }
  }
  // the slice's offset within its first chunk is uniform: one branch, register moves
#define NCA_SLICE_AT(D)                                                                        \
  case D:                                                                                      \
    _Pragma("unroll") for (int c = 0; c < MAXC; ++c) xs[c] = v[(c + D) < S::NK * S::CW ? c + D : 0]; \
    break;
  switch (d) {
    NCA_SLICE_AT(0) NCA_SLICE_AT(1) NCA_SLICE_AT(2) NCA_SLICE_AT(3)
    NCA_SLICE_AT(4) NCA_SLICE_AT(5) NCA_SLICE_AT(6) NCA_SLICE_AT(7)
  }
#undef NCA_SLICE_AT
#pragma unroll
  for (int c = 0; c < MAXC; ++c) xs[c] = c < A.c_out ? xs[c] : 0.f;
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1) nca_step_kernel(const __grid_constant__ StepArgs A) {
  using namespace nca;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const SmemLayout<Cfg> L(A.stages, A.win_cells, A.wimg_lo != nullptr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L.misc);
  int* abort_flag = reinterpret_cast<int*>(smem + L.misc + 8);
  // epilogue warps that have stored a tile (8 per tile), read by the publisher lane
  unsigned* s_tiles_done = reinterpret_cast<unsigned*>(smem + L.misc + 16);
  float* s_b1 = reinterpret_cast<float*>(smem + L.b1);
  float* s_b2 = reinterpret_cast<float*>(smem + L.b2);
  uint8_t* s_flags = smem + L.flags;  // [4][128]: bit0 fire, bit1 given, bit2 valid

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  FailState fs;
  fs.ctrl = A.ctrl;
  fs.cta_abort = abort_flag;
  fs.timeout_ns = A.timeout_ns;
  fs.deadline_ns = 0;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    *s_tiles_done = 0;
    for (int s = 0; s < kMaxStages; ++s) {
      mbar_init(&bars[BAR_WIN_FULL + s], 1);
      // released by the 8 stencil warps, or in the hi/lo layout by the epilogue warps, which
      // read the hi part of the old state from the window
      mbar_init(&bars[BAR_WIN_EMPTY + s], Cfg::HILO ? Cfg::EPI_WARPS : 8);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[BAR_Z_FULL + s], 8);
      mbar_init(&bars[BAR_Z_EMPTY + s], 1);
    }
    for (int r = 0; r < 2; ++r) {
      mbar_init(&bars[BAR_ACC_FULL + r], 1);
      mbar_init(&bars[BAR_ACC_FULL_B + r], 1);
      mbar_init(&bars[BAR_H_FULL + r], 4 * Cfg::PARTS_PER_HALF);
      mbar_init(&bars[BAR_H_FULL_B + r], 4 * Cfg::PARTS_PER_HALF);
      mbar_init(&bars[BAR_ACC2_FULL + r], 1);
      mbar_init(&bars[BAR_ACC_EMPTY + r], Cfg::EPI_WARPS);
    }
    mbar_init(&bars[BAR_WEIGHTS], 1);
    mbar_init(&bars[BAR_DRAIN], 1);
    // the flags of a tile come from the 4 half-0 stencil warps
    for (int r = 0; r < 4; ++r) mbar_init(&bars[BAR_FLAGS + r], 4);
    for (int r = 0; r < 8; ++r) mbar_init(&bars[BAR_PAIR + r], 1);
    mbar_init(&bars[BAR_RES_LOADED], Cfg::EPI_WARPS);
    for (int i = 0; i < 8; ++i) reinterpret_cast<unsigned*>(smem + L.misc + 32)[i] = 0u;
    fence_mbar_init();
  }
  // Every chunk row of a window stage ends with a padding cell (index win_cells): the stencil
  // reads it for neighbours outside the board, so no load is predicated.
  for (int i = threadIdx.x; i < A.stages * Cfg::NCH; i += Cfg::THREADS) {
    const int stg = i / Cfg::NCH, ch = i % Cfg::NCH;
    uint8_t* cell = smem + L.win + (stg * (A.win_cells + 1) * Cfg::NCH + ch * (A.win_cells + 1) + A.win_cells) * 16;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if constexpr (Cfg::SRC_BF16) {
        w[e] = pack_bf16(A.pad[ch * 8 + 2 * e], A.pad[ch * 8 + 2 * e + 1]);
      } else {
        w[e] = __float_as_uint(A.pad[ch * 4 + e]);
      }
    }
    *reinterpret_cast<uint4*>(cell) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  for (int i = threadIdx.x; i < Cfg::HD; i += Cfg::THREADS) s_b1[i] = A.b1[i];
  for (int i = threadIdx.x; i < Cfg::C; i += Cfg::THREADS) s_b2[i] = A.b2[i];
  if (warp == 0) {
    tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // A previous launch on this control block failed: do not touch the state.
  const bool skip = (*((volatile int*)&A.ctrl[0]) != 0);
  const int wg = warp >> 2;

  const int grid = gridDim.x;
  const long long total = A.total;
  const int W = A.W;

  if (!skip && wg == 0) {
  if (warp == 0) {
    // ---------------------------------------------------------------- MMA issuer
    if (Cfg::TILEDEP && lane == 1 && A.n_steps > 1) {
      // ------------------------------------------------------------ publisher
      // In tile order: once the epilogue warps have stored tile t of step s, a gpu-scope
      // fence (cumulative over those stores, acquired at CTA scope) and the tile's counter
      // tile_steps[t] = s + 1, which the loaders of neighbouring tiles wait for.
      uint32_t it = 0;
      bool ok = true;
      for (int s = 0; ok && s + 1 < A.n_steps; ++s) {
        for (long long t = blockIdx.x; t < A.n_tiles; t += grid, ++it) {
          const unsigned want = (unsigned)(Cfg::EPI_WARPS + (Cfg::ADAPTIVE ? 2 : 0)) * (unsigned)(it + 1);
          uint64_t start = 0;
          for (uint32_t k = 0;; ++k) {
            unsigned v;
            asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(s_tiles_done)) : "memory");
            if (v >= want) break;
            if ((k & 63) == 63) {
              const uint64_t now = global_timer_ns();
              if (start == 0) start = now;
              if (should_abort(fs)) { ok = false; break; }
              if (now - start > fs.timeout_ns || k > (1u << 28)) {
                report_failure(fs, 4, W_PUBLISH);
                ok = false;
                break;
              }
            }
            __nanosleep(32);
          }
          if (!ok) break;
          __threadfence();
          asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(A.tile_steps + t), "r"((unsigned)(s + 1)) : "memory");
        }
        // this CTA has stored every tile of step s
        if (ok) atomicAdd(reinterpret_cast<unsigned*>(A.ctrl + 2), 1u);
      }
    }
    if (lane == 0) {
      bool ok = true;
      // weights are loaded by the loader warp
      {
        uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&bars[BAR_WEIGHTS], 0)) {
          if (should_abort(fs)) { ok = false; break; }
          if (global_timer_ns() - t0 > fs.timeout_ns) { report_failure(fs, 4, W_MMA_WEIGHTS); ok = false; break; }
          __nanosleep(64);
        }
      }
      const uint32_t w1 = smem_u32(smem + L.w1);
      const uint32_t w2 = smem_u32(smem + L.w2);
      const uint32_t id1 = idesc_bf16_f32(kTileM, Cfg::HD / 2);
      const uint64_t d1 = umma_desc_sw128(w1);
      const uint64_t d2 = umma_desc_sw128(w2);
      const uint32_t id2 = idesc_bf16_f32(kTileM, Cfg::C);
      // split mode with fp32 weights: the residual image adds z_hi * W_lo (and h_hi * W2_lo)
      const bool wlo = Cfg::SPLIT && A.wimg_lo != nullptr;
      const uint64_t d1lo = umma_desc_sw128(smem_u32(smem + L.w1lo));
      const uint64_t d2lo = umma_desc_sw128(smem_u32(smem + L.w2lo));
      uint32_t it = 0;
      const long long n_pass = pass_count<Cfg>(A, grid);
      for (long long ps = 0; ok && ps < n_pass; ++ps) {
      const Pass P = pass_of<Cfg>(A, ps, grid);
      for (int s = 0; ok && s < A.n_steps; ++s) {
        for (long long t = P.t0; ok && t < P.t1; t += P.dt, ++it) {
          const int slot = (int)(it % Cfg::NZ);
          const uint32_t u = (uint32_t)(it / Cfg::NZ);
          const uint32_t zcol = tmem + slot * Cfg::SLOT_COLS;
          const int rg = (int)(it % Cfg::NACC);             // accumulator region
          const uint32_t ua = (uint32_t)(it / Cfg::NACC) & 1;  // its phase
          const uint32_t acol = tmem + Cfg::ACC_COL + rg * Cfg::HD;
          const uint32_t a2col = acol + (Cfg::ACC2_COL - Cfg::ACC_COL);
          if (!mbar_wait(&bars[BAR_Z_FULL + slot], u & 1, fs, W_MMA_ZFULL)) { ok = false; break; }
          if (!mbar_wait(&bars[BAR_ACC_EMPTY + rg], ua ^ 1, fs, W_MMA_ACCEMPTY)) { ok = false; break; }
          tc_fence_after();
          // GEMM1 in two N halves (hidden units [0, HD/2) then [HD/2, HD)).  In bf16 mode each half
          // is committed on its own, so that the hidden epilogue of the first half overlaps the
          // second half, and the z slot is released right after GEMM1.  The loops are unrolled
          // and every descriptor is a constant offset of d1/d2, so one thread issues the MMAs
          // faster than the tensor core retires them.
#pragma unroll
          for (int nh = 0; nh < 2; ++nh) {
#pragma unroll
            for (int kk = 0; kk < Cfg::P / 16; ++kk) {
              const uint32_t boff = (kk >> 2) * (Cfg::HD * 128) + nh * (Cfg::HD / 2) * 128 + (kk & 3) * 32;
#pragma unroll
              for (int part = 0; part < Cfg::ZPARTS; ++part)
                umma_bf16_ts(acol + nh * (Cfg::HD / 2), zcol + part * (Cfg::P / 2) + kk * 8,
                             desc_add(d1, boff), id1, (kk | part) != 0);
              if (Cfg::SPLIT && wlo)
                umma_bf16_ts(acol + nh * (Cfg::HD / 2), zcol + kk * 8, desc_add(d1lo, boff), id1, 1u);
            }
            if (Cfg::H_IN_ACC) umma_commit(&bars[(nh == 0 ? BAR_ACC_FULL : BAR_ACC_FULL_B) + rg]);
          }
          if (Cfg::H_IN_ACC) {
            umma_commit(&bars[BAR_Z_EMPTY + slot]);
          } else {
            umma_commit(&bars[BAR_ACC_FULL + rg]);
            umma_commit(&bars[BAR_ACC_FULL_B + rg]);
          }
          // GEMM2 in two K halves, each as soon as its half of h is in tensor memory.
#pragma unroll
          for (int kh = 0; kh < 2; ++kh) {
            if (!mbar_wait(&bars[(kh == 0 ? BAR_H_FULL : BAR_H_FULL_B) + rg], ua, fs, W_MMA_HFULL)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int kq = 0; kq < Cfg::HD / 32; ++kq) {
              const int kk = kh * (Cfg::HD / 32) + kq;
              const uint32_t boff = (kk >> 2) * (Cfg::C * 128) + (kk & 3) * 32;
              if constexpr (Cfg::H_IN_ACC) {
                umma_bf16_ts(a2col, acol + kh * (Cfg::HD / 2) + kq * 8, desc_add(d2, boff), id2, kk != 0);
              } else {
#pragma unroll
                for (int part = 0; part < Cfg::ZPARTS; ++part)
                  umma_bf16_ts(a2col, zcol + part * (Cfg::HD / 2) + kk * 8, desc_add(d2, boff), id2,
                               (kk | part) != 0);
                if (wlo) umma_bf16_ts(a2col, zcol + kk * 8, desc_add(d2lo, boff), id2, 1u);
              }
            }
          }
          if (!ok) break;
          umma_commit(&bars[BAR_ACC2_FULL + rg]);
          if (!Cfg::H_IN_ACC) umma_commit(&bars[BAR_Z_EMPTY + slot]);
        }
      }
      }  // passes
      // Drain: every MMA issued above has completed once this commit arrives.
      umma_commit(&bars[BAR_DRAIN]);
      uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&bars[BAR_DRAIN], 0)) {
        if (global_timer_ns() - t0 > fs.timeout_ns) { report_failure(fs, 4, W_DRAIN); break; }
        __nanosleep(64);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- loader
    if (lane == 0) {
      const int tot = Cfg::W1_BYTES + Cfg::W2_BYTES;   // w1 and w2 are contiguous in smem
      mbar_arrive_expect_tx(&bars[BAR_WEIGHTS], A.wimg_lo ? 2 * tot : tot);
      const uint32_t dst = smem_u32(smem + L.w1);
      for (int off = 0; off < tot; off += 16384) {
        const int n = (tot - off) < 16384 ? (tot - off) : 16384;
        bulk_g2s(dst + off, A.wimg + off, n, &bars[BAR_WEIGHTS]);
      }
      if (A.wimg_lo) {
        const uint32_t dlo = smem_u32(smem + L.w1lo);
        for (int off = 0; off < tot; off += 16384) {
          const int n = (tot - off) < 16384 ? (tot - off) : 16384;
          bulk_g2s(dlo + off, A.wimg_lo + off, n, &bars[BAR_WEIGHTS]);
        }
      }
    }
    __syncwarp();
    const int NCH = Cfg::NCH;
    const int WC = A.win_cells;
    const int S = A.stages;
    int stage = 0;      // window stage of the current tile: it % S, kept incrementally
    uint32_t vph = 0;   // (it / S) & 1
    uint32_t it = 0;
    bool ok = true;
    int done_step = 0;  // every tile has stored the steps before done_step
    // (resident mode: no windows; the epilogue warps load each group's state)
    for (int s = 0; ok && !Cfg::RESIDENT && s < A.n_steps; ++s) {
      const int in = (A.cur + s) & 1;
      const uint8_t* src = Cfg::SRC_BF16 ? reinterpret_cast<const uint8_t*>(A.mirror[in])
                                         : reinterpret_cast<const uint8_t*>(A.master[in]);
      if (!Cfg::TILEDEP && s > 0) {
        // grid barrier: every CTA has stored its tiles of step s-1
        int give_up = 0;
        if (lane == 0) {
          const unsigned target = (unsigned)s * (unsigned)grid;
          uint64_t t0 = global_timer_ns();
          for (uint32_t k = 0;; ++k) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(&A.ctrl[2]) : "memory");
            if (v >= target) break;
            if (should_abort(fs)) { give_up = 1; break; }
            if (global_timer_ns() - t0 > fs.timeout_ns || k > (1u << 28)) {
              report_failure(fs, 4, W_LOAD_GRID);
              give_up = 1;
              break;
            }
            __nanosleep(128);
          }
        }
        if (__shfl_sync(0xffffffffu, give_up, 0)) { ok = false; break; }
      }
      for (long long t = blockIdx.x; t < A.n_tiles;
           t += grid, ++it, stage = (stage + 1 == S ? 0 : stage + 1), vph ^= (stage == 0 ? 1u : 0u)) {
        const uint32_t v = vph;  // parity of the stage's use
        if (!warp_wait(&bars[BAR_WIN_EMPTY + stage], (v & 1) ^ 1, fs, W_LOAD_EMPTY)) { ok = false; break; }
        const long long wb = t * kTileM - W - 1;
        const long long lo = wb < 0 ? 0 : wb;
        const long long hi = (wb + WC) < total ? (wb + WC) : total;
        if (Cfg::TILEDEP && s > 0 && done_step < s) {
          // Per-tile dependencies instead of a grid barrier: the window reads step s-1 of the
          // tiles it overlaps, so each of them must have stored step s-1 (their counters reach s).
          // The same condition orders this tile's later stores into the other buffer after
          // those tiles' reads of it at step s-1.  One lane per overlapped tile, bounded; lane 31
          // also reads the count of CTAs that finished step s-1 (ctrl[2]), and once every CTA
          // has, the rest of the step needs no checks.
          const long long T = (lo >> 7) + lane;
          bool need = T <= ((hi - 1) >> 7);
          uint64_t start = 0;
          for (uint32_t k = 0;; ++k) {
            if (need) {
              unsigned v;
              asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(A.tile_steps + T) : "memory");
              need = v < (unsigned)s;
            }
            unsigned all = 0;
            if (lane == 31) {
              unsigned v;
              asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(A.ctrl + 2) : "memory");
              all = v >= (unsigned)s * (unsigned)grid ? 1u : 0u;
            }
            if (__shfl_sync(0xffffffffu, all, 31)) {
              done_step = s;
              break;
            }
            if (!__any_sync(0xffffffffu, need)) break;
            int give_up = 0;
            if (lane == 0 && (k & 15) == 15) {
              const uint64_t now = global_timer_ns();
              if (start == 0) start = now;
              if (should_abort(fs)) give_up = 1;
              else if (now - start > fs.timeout_ns || k > (1u << 28)) {
                report_failure(fs, 4, W_LOAD_GRID);
                give_up = 1;
              }
            }
            if (__shfl_sync(0xffffffffu, give_up, 0)) { ok = false; break; }
            __nanosleep(64);
          }
          if (!ok) break;
        }
        if (lane == 0)
          mbar_arrive_expect_tx(&bars[BAR_WIN_FULL + stage],
                                (uint32_t)(NCH * (hi - lo) * 16) + (Cfg::ADAPTIVE ? kTileM * 4u : 0u));
        __syncwarp();
        if constexpr (Cfg::ADAPTIVE) {
          // the fire probabilities of the tile's cells for this step (written by the epilogue at
          // the previous step, or before the launch)
          if (lane == 31)
            bulk_g2s(smem_u32(smem + L.pwin + stage * kTileM * 4), A.fire_p + t * kTileM, kTileM * 4,
                     &bars[BAR_WIN_FULL + stage]);
        }
        const uint32_t dst = smem_u32(smem + L.win + stage * (WC + 1) * Cfg::ROWB);
        // one bulk copy per (chunk, tile overlapped by the window): 3 tiles while the board is
        // narrower than a tile, up to 2 + ceil((2W + 2) / 128) for wider boards
        const long long t0 = lo >> 7;
        const int nt = (int)(((hi - 1) >> 7) - t0 + 1);
        for (int job = lane; job < NCH * nt; job += 32) {
          const int ch = job / nt;
          const long long T = t0 + job % nt;
          const long long c_lo = (T << 7) > lo ? (T << 7) : lo;
          const long long c_hi = ((T + 1) << 7) < hi ? ((T + 1) << 7) : hi;
          if (c_hi > c_lo) {
            const uint8_t* p = src + (((T * NCH + ch) << 7) + (c_lo & 127)) * 16;
            bulk_g2s(dst + (uint32_t)((ch * (WC + 1) + (c_lo - wb)) * 16), p, (uint32_t)((c_hi - c_lo) * 16),
                     &bars[BAR_WIN_FULL + stage]);
          }
        }
        // The part of the tile's old state that the epilogue reads from global memory (the lo
        // parts in the hi/lo layout, else the fp32 state; the adaptive rule reads it too): into
        // L2 now, a few tiles before the epilogue's loads.
        if (lane == 0)
          bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(A.master[in]) + t * kTileM * Cfg::C * (Cfg::HILO ? 2 : 4),
                           kTileM * Cfg::C * (Cfg::HILO ? 2 : 4));
      }
    }
    // Bulk copies still in flight (only after an abort) must land before the CTA exits.
    if (lane == 0) {
      for (int sg = 0; sg < S && sg < it; ++sg) {
        const long long last = ((it - 1 - sg) / S) * S + sg;  // last tile index issued on stage sg
        const uint32_t par = (uint32_t)(last / S) & 1;
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&bars[BAR_WIN_FULL + sg], par)) {
          if (global_timer_ns() - t0 > fs.timeout_ns) { report_failure(fs, 4, W_DRAIN); break; }
        }
      }
    }
    __syncwarp();
  } else if (Cfg::ADAPTIVE) {
    // ---------------------------------------------------------------- confidence (warps 2, 3)
    // Adaptive rules: per tile, once every epilogue warp has stored the tile's new state (their
    // progress words), the readout slice of each row is read back from global memory (L2) ->
    // the head -> the cell's fire probability of the next step, 2 rows per lane.  The epilogue
    // never waits for these warps within a step; their stores count for the step end like the
    // epilogue's.
    const int cw = warp - 2;
    const unsigned* s_prog = reinterpret_cast<const unsigned*>(smem + L.misc + 32);
    float* s_head = reinterpret_cast<float*>(smem + L.head) + cw * kHeadFloats;
    for (int i = lane; i < kHeadFloats; i += 32) s_head[i] = i < 256 ? A.head_w[i >> 4][i & 15] : A.head_b[i - 256];
    __syncwarp();
    // Each warp evaluates rows cw * 64 + lane and cw * 64 + 32 + lane of every tile: the loads of
    // both rows are issued before either is used.  Fast path (mlp head, c_out <= 9, n_out <= 10):
    // 9 channels per row, the head row by row; the general head keeps 16 channels per row.
    uint32_t it = 0;
    bool ok = true;
    auto conf_loop = [&](auto maxc_tag) {
      constexpr int MAXC = decltype(maxc_tag)::value;
      struct Row {
        SliceRaw<Cfg, MAXC> raw;
        unsigned g;  // global cell
        int given;   // the cell's given byte
      };
      // the given bytes of a tile's two rows: static data, loaded a tile ahead of their use
      auto load_given = [&](long long t, int (&gv)[2]) {
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const unsigned g = (unsigned)(t * kTileM) + (unsigned)(cw * 64 + rr * 32 + lane);
          gv[rr] = 0;
          if (t < A.n_tiles && (long long)g < total) {
            const int inst = (int)fdiv(g, A.div_hw);
            const int p = (int)(g - (unsigned)inst * A.HW);
            const int row = A.inst_row ? A.inst_row[inst] : (int)fdiv((unsigned)inst, A.div_k);
            gv[rr] = A.given[(long long)row * A.HW + p];
          }
        }
      };
      auto issue = [&](Row& R, long long t, int out, int rr, int given) {
        const int r = cw * 64 + rr * 32 + lane;
        slice_issue<Cfg, MAXC>(A, out, t, r, R.raw);
        R.g = (unsigned)(t * kTileM) + (unsigned)r;
        R.given = given;
      };
      auto store = [&](const Row& R, float conf) {
        if ((long long)R.g < total)
          A.fire_p[R.g] = adaptive_prob(A.fire_mode, conf, R.given != 0, A.ad_scale, A.ad_bias, A.p_low,
                                        A.tau, A.p_fire, A.given_confident);
      };
      auto tile_done = [&]() {
        if constexpr (Cfg::TILEDEP) {
          __syncwarp();
          if (lane == 0) asm volatile("red.release.cta.shared::cta.add.u32 [%0], 1;" ::"r"(smem_u32(s_tiles_done)) : "memory");
        }
      };
      auto finish1 = [&](const Row& R) {
        float x[1][MAXC], conf[1];
        slice_values<Cfg, MAXC>(A, R.raw, x[0]);
        head_confidence<MAXC, 10, 1>(A.n_out, s_head, x, conf);
        store(R, conf[0]);
      };
      Row ra, rb;
      int gnext[2];
      for (int s = 0; ok && s < A.n_steps; ++s) {
        const int out = (A.cur + s + 1) & 1;
        load_given(blockIdx.x, gnext);
        for (long long t = blockIdx.x; t < A.n_tiles; t += grid, ++it) {
          const int g0 = gnext[0], g1 = gnext[1];
          load_given(t + grid, gnext);
          if (!wait_progress(s_prog, Cfg::EPI_WARPS, it + 1u, fs, W_CONF)) { ok = false; break; }
          issue(ra, t, out, 0, g0);
          issue(rb, t, out, 1, g1);
          if constexpr (MAXC == 9) {
            finish1(ra);
            finish1(rb);
            tile_done();
          } else {
            float x[2][MAXC], conf[2];
            slice_values<Cfg, MAXC>(A, ra.raw, x[0]);
            slice_values<Cfg, MAXC>(A, rb.raw, x[1]);
            if (A.head_kind != 0) {
#pragma unroll
              for (int rr = 0; rr < 2; ++rr) {
                int arg;
                head_readout_auto(A.head_kind, A.n_out, A.c_out, A.head_w, A.head_b, x[rr], conf[rr], arg);
              }
            } else {
              head_confidence<16, 16, 2>(A.n_out, s_head, x, conf);
            }
            store(ra, conf[0]);
            store(rb, conf[1]);
            tile_done();
          }
        }
        if constexpr (!Cfg::TILEDEP) {
          // the step end of the epilogue warps, joined by these two warps (their stores of the step
          // are then covered by the epilogue's fence before the step counter)
          unsigned any_fail;
          asm volatile(
              "{\n\t.reg .pred p, q;\n\t"
              "setp.ne.u32 p, %1, 0;\n\t"
              "bar.red.or.pred q, 1, %2, p;\n\t"
              "selp.u32 %0, 1, 0, q;\n\t}"
              : "=r"(any_fail)
              : "r"((unsigned)(!ok || *(volatile int*)abort_flag != 0)), "n"(Cfg::EPI_WARPS * 32 + 64)
              : "memory");
          if (any_fail) { ok = false; break; }
        }
      }
    };
    if (A.head_kind == 0 && A.c_out <= 9 && A.n_out <= 10) conf_loop(IntTag<9>{});
    else conf_loop(IntTag<16>{});
  }  // without the adaptive rules, warps 2 and 3 are idle
  } else if (!skip && warp >= kStencilWarp0 && warp < kEpiWarp0) {
    // ---------------------------------------------------------------- stencil
    const int sw = warp - kStencilWarp0;
    const int half = sw >> 2;
    const int quarter = warp & 3;
    const int m = quarter * 32 + lane;     // tile row = TMEM lane
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int WC = A.win_cells;
    const int S = A.stages;
    int stage = 0;      // window stage of the current tile: it % S, kept incrementally
    uint32_t vph = 0;   // (it / S) & 1
    uint32_t it = 0;
    bool ok = true;
    const long long n_pass = pass_count<Cfg>(A, grid);
    const unsigned* s_prog = reinterpret_cast<const unsigned*>(smem + L.misc + 32);
    for (long long ps = 0; ok && ps < n_pass; ++ps) {
    const Pass P = pass_of<Cfg>(A, ps, grid);
    for (int s = 0; ok && s < A.n_steps; ++s) {
      for (long long t = P.t0; t < P.t1;
           t += P.dt, ++it, stage = (stage + 1 == S ? 0 : stage + 1), vph ^= (stage == 0 ? 1u : 0u)) {
        const uint32_t v = vph;  // parity of the stage's use
        const int slot = (int)(it % Cfg::NZ);
        const uint32_t u = (uint32_t)(it / Cfg::NZ);
        // Index math and the per-row side information for the epilogue come before the waits
        // (they depend only on the cell and the step, and their global loads then overlap the
        // wait for the window): bit 0 the fire decision of this step, bit 1 given, bit 2 valid
        // (the adaptive rules are evaluated after z, below).
        const unsigned g = (unsigned)(P.cell0 + t * kTileM) + m;
        const bool valid = (long long)g < P.lim;
        int i = 0, j = 0, inst = 0, p = 0;
        if (valid) {
          inst = (int)fdiv(g, A.div_hw);
          p = (int)(g - (unsigned)inst * A.HW);
          i = (int)fdiv((unsigned)p, A.div_w);
          j = p - i * W;
        }
        uint32_t fl = 0;
        float ufire = 0.f;  // adaptive rules: the uniform the cell's fire probability is drawn against
        if (half == 0 && valid) {
          const int row = A.inst_row ? A.inst_row[inst] : (int)fdiv((unsigned)inst, A.div_k);
          fl = 4u | (A.given[(long long)row * A.HW + p] ? 2u : 0u);
          if constexpr (Cfg::ADAPTIVE) {
            ufire = (A.fire_mode == 3 || A.fire_mode == 5)
                        ? A.uniforms[((long long)s * A.n_inst + inst) * A.HW + p]
                        : philox_uniform(A.seed, A.inst_offset + (A.inst_id ? A.inst_id[inst] : inst), p, A.step0 + s);
          } else if (A.fire_mode == 0) {
            fl |= A.masks[((long long)s * A.n_inst + inst) * A.HW + p] ? 1u : 0u;
          } else {
            fl |= philox_uniform(A.seed, A.inst_offset + (A.inst_id ? A.inst_id[inst] : inst), p, A.step0 + s) < A.p_fire ? 1u : 0u;
          }
        }
        if constexpr (Cfg::RESIDENT) {
          // The hi parts of step s are in buffer s & 1: at the group's first step the epilogue's
          // load of the group; later the previous step's epilogue of this tile and its
          // neighbours (up to tile t + 1), which every epilogue warp reports in its progress word.
          if (s == 0) {
            if (t == 0 && !warp_wait(&bars[BAR_RES_LOADED], (uint32_t)ps & 1, fs, W_RES)) { ok = false; break; }
          } else {
            const long long tn = t + 1 < P.t1 ? t + 1 : P.t1 - 1;
            const unsigned need = it - (unsigned)(t + P.t1) + (unsigned)tn + 1u;  // it of (s-1, tn), + 1
            if (!wait_progress(s_prog, Cfg::EPI_WARPS, need, fs, W_RES)) { ok = false; break; }
          }
        } else {
          if (!warp_wait(&bars[BAR_WIN_FULL + stage], v & 1, fs, W_ST_WINFULL)) { ok = false; break; }
        }
        if (!warp_wait(&bars[BAR_Z_EMPTY + slot], (u & 1) ^ 1, fs, W_ST_ZEMPTY)) { ok = false; break; }
        tc_fence_after();
        const uint8_t* win = smem + L.win + (Cfg::RESIDENT ? (s & 1) : stage) * (WC + 1) * Cfg::ROWB;
        if (half == 0) {
          if constexpr (Cfg::ADAPTIVE) {
            // the cell's fire probability of this step, copied with the window
            const float pf = reinterpret_cast<const float*>(smem + L.pwin + stage * kTileM * 4)[m];
            fl |= (valid && ufire < pf) ? 1u : 0u;
          }
          s_flags[(it & 3) * kTileM + m] = (uint8_t)fl;
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[BAR_FLAGS + (it & 3)]);
          if (!Cfg::RESIDENT && !Cfg::TILEDEP && A.updates != nullptr) {
            // Fired cells per instance.  With the grid barrier these warps have slack (they wait
            // for windows) while the epilogue is on the tile's critical path, so they count;
            // the resident form and per-tile step counters count in the epilogue instead
            // (measured either way).
            const unsigned grp = __match_any_sync(0xffffffffu, valid ? inst : -1);
            const unsigned fm = __ballot_sync(0xffffffffu, (fl & 1u) != 0);
            if (valid && lane == __ffs(grp) - 1) {
              const int cnt = __popc(fm & grp);
              if (cnt) atomicAdd(&A.updates[inst], (unsigned)cnt);
            }
          }
        }
        const bool up = valid && i > 0, dn = valid && i < A.H - 1;
        const bool lf = valid && j > 0, rt = valid && j < W - 1;
        // window index of this cell (resident: its index in the group)
        const int c0 = Cfg::RESIDENT ? (int)(t * kTileM) + m : m + W + 1;
        const uint32_t zbase = tmem + lane_addr + slot * Cfg::SLOT_COLS;
        // the 9 neighbours a b c / d e f / g h k: their cell offsets in the window stage
        const uint32_t wbase = smem_u32(win);
        uint32_t nb_row[9];
        bool nb_ok[9];
#pragma unroll
        for (int n = 0; n < 9; ++n) {
          const int dy = n / 3 - 1, dx = n % 3 - 1;
          const int wc = c0 + dy * W + dx;
          nb_ok[n] = (dy < 0 ? up : (dy > 0 ? dn : valid)) && (dx < 0 ? lf : (dx > 0 ? rt : true));
          nb_row[n] = wbase + (uint32_t)(nb_ok[n] ? wc : WC) * 16u;  // WC: the padding cell
        }
#pragma unroll 1
        for (int q = 0; q < Cfg::NCH / 2; ++q) {
          const int ch = half * (Cfg::NCH / 2) + q;
          const uint32_t choff = (uint32_t)(ch * (WC + 1)) * 16u;
          uint4 v[9];
#pragma unroll
          for (int n = 0; n < 9; ++n)
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(v[n].x), "=r"(v[n].y), "=r"(v[n].z), "=r"(v[n].w)
                         : "r"(nb_row[n] + choff));
          if constexpr (Cfg::SRC_BF16) {
            // 8 channels ch*8 .. ch*8+7 as 4 bf16 pairs; identity, Sobel-x, Sobel-y, Laplacian
            uint32_t zi[4], zx[4], zy[4], zl[4];
            if (A.fixed_taps) {
              // packed bf16x2 arithmetic (two channels per instruction, each operation rounded to
              // bf16): column sums S = top + 2 mid + bottom and differences D = bottom - top of the
              // left, middle and right columns give the three heads.
              const __nv_bfloat162 two = __float2bfloat162_rn(2.f), k8 = __float2bfloat162_rn(0.125f);
              const __nv_bfloat162 k16 = __float2bfloat162_rn(0.0625f), m16 = __float2bfloat162_rn(-16.f);
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                auto B2 = [&](int n) { return *reinterpret_cast<const __nv_bfloat162*>(&v[n].x + w); };
                const __nv_bfloat162 a = B2(0), b = B2(1), c = B2(2), d = B2(3), e = B2(4);
                const __nv_bfloat162 f = B2(5), g = B2(6), h = B2(7), k = B2(8);
                const __nv_bfloat162 sl = __hadd2(__hfma2(two, d, a), g);
                const __nv_bfloat162 sm = __hadd2(__hfma2(two, e, b), h);
                const __nv_bfloat162 sr = __hadd2(__hfma2(two, f, c), k);
                const __nv_bfloat162 dl = __hsub2(g, a), dm = __hsub2(h, b), dr = __hsub2(k, c);
                const __nv_bfloat162 sx = __hmul2(__hsub2(sr, sl), k8);
                const __nv_bfloat162 sy = __hmul2(__hadd2(__hfma2(two, dm, dl), dr), k8);
                const __nv_bfloat162 lp = __hmul2(__hfma2(m16, e, __hadd2(__hfma2(two, sm, sl), sr)), k16);
                zi[w] = (&v[4].x)[w];  // identity head of a bf16 source is the value itself
                zx[w] = *reinterpret_cast<const uint32_t*>(&sx);
                zy[w] = *reinterpret_cast<const uint32_t*>(&sy);
                zl[w] = *reinterpret_cast<const uint32_t*>(&lp);
              }
            } else {
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                float o[4][2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  float nb[9];
#pragma unroll
                  for (int n = 0; n < 9; ++n) {
                    const uint32_t x = (&v[n].x)[w];
                    nb[n] = e == 0 ? bf16lo_to_f32(x) : bf16hi_to_f32(x);
                  }
#pragma unroll
                  for (int kh = 0; kh < 4; ++kh) {
                    float acc = 0.f;
#pragma unroll
                    for (int n = 0; n < 9; ++n) acc = fmaf(A.taps[kh][n], nb[n], acc);
                    o[kh][e] = acc;
                  }
                }
                zi[w] = pack_bf16(o[0][0], o[0][1]);
                zx[w] = pack_bf16(o[1][0], o[1][1]);
                zy[w] = pack_bf16(o[2][0], o[2][1]);
                zl[w] = pack_bf16(o[3][0], o[3][1]);
              }
            }
            const int cb = ch * 8;  // first channel of the chunk
            tmem_st4(zbase + (0 * Cfg::C + cb) / 2, zi);
            tmem_st4(zbase + (1 * Cfg::C + cb) / 2, zx);
            tmem_st4(zbase + (2 * Cfg::C + cb) / 2, zy);
            tmem_st4(zbase + (3 * Cfg::C + cb) / 2, zl);
          } else {
            // fp32 source, 4 channels: ch*4 .. ch*4+3; z split into bf16 hi + lo parts
            float z[4][4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float nb[9];
#pragma unroll
              for (int n = 0; n < 9; ++n) nb[n] = __uint_as_float((&v[n].x)[e]);
              if (A.fixed_taps) {
                z[0][e] = nb[4];
                fixed_taps4(nb[0], nb[1], nb[2], nb[3], nb[4], nb[5], nb[6], nb[7], nb[8], z[1][e],
                            z[2][e], z[3][e]);
              } else {
#pragma unroll
                for (int kh = 0; kh < 4; ++kh) {
                  float acc = 0.f;
#pragma unroll
                  for (int n = 0; n < 9; ++n) acc = fmaf(A.taps[kh][n], nb[n], acc);
                  z[kh][e] = acc;
                }
              }
            }
            const int cb = ch * 4;
#pragma unroll
            for (int kh = 0; kh < 4; ++kh) {
              const uint32_t h01 = pack_bf16(z[kh][0], z[kh][1]);
              const uint32_t h23 = pack_bf16(z[kh][2], z[kh][3]);
              const uint32_t l01 = pack_bf16(z[kh][0] - bf16lo_to_f32(h01), z[kh][1] - bf16hi_to_f32(h01));
              const uint32_t l23 = pack_bf16(z[kh][2] - bf16lo_to_f32(h23), z[kh][3] - bf16hi_to_f32(h23));
              const uint32_t col = (kh * Cfg::C + cb) / 2;
              tmem_st2(zbase + col, h01, h23);
              tmem_st2(zbase + Cfg::P / 2 + col, l01, l23);
            }
          }
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_relaxed(&bars[BAR_Z_FULL + slot]);
          // hi/lo layout: the epilogue still reads the tile's own cells (the hi part of the old
          // state) from this window and releases it
          if constexpr (!Cfg::HILO && !Cfg::RESIDENT) mbar_arrive_relaxed(&bars[BAR_WIN_EMPTY + stage]);
        }
      }
    }
    }  // passes
  } else if (!skip && warp >= kEpiWarp0) {
    // ---------------------------------------------------------------- epilogue
    // Part p of the epilogue (EPI_PARTS warps per lane quarter): E1 of the hidden units
    // [p * HPART, (p + 1) * HPART), which lie in GEMM1 N-half hh, and E2 of the channels
    // [p * CH, (p + 1) * CH).
    const int ew = warp - kEpiWarp0;
    const int part = ew >> 2;
    const int hh = part / Cfg::PARTS_PER_HALF;
    const int sub = part % Cfg::PARTS_PER_HALF;
    const int quarter = warp & 3;
    const int m = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    constexpr int CH = Cfg::CH;             // channels of this thread in E2
    constexpr int HPART = Cfg::HD / Cfg::EPI_PARTS;
    // columns per tensor-memory load in split mode's E1 (it writes hi and lo parts)
    constexpr int E1C = 16;
    // bf16 mode writes h over accumulator columns already read: the second part of a half
    // writes into the first part's columns, after that part's reads (BAR_PAIR of the lane
    // quarter and half, one phase per tile)
    uint64_t* pair_bar = &bars[BAR_PAIR + quarter + 4 * hh];
    uint32_t it = 0;
    int wstage = 0;  // window stage of the current tile (it % stages)
    bool ok = true;
    const long long n_pass = pass_count<Cfg>(A, grid);
    unsigned* s_prog = reinterpret_cast<unsigned*>(smem + L.misc + 32);  // resident: per-warp progress
    for (long long ps = 0; ok && ps < n_pass; ++ps) {
    const Pass P = pass_of<Cfg>(A, ps, grid);
    if constexpr (Cfg::RESIDENT) {
      // The group's state into shared memory (hi parts to buffer 0, lo parts).  Every epilogue
      // warp is done with the previous group (the barrier at the end of each pass), and the
      // stencil finished with it before the epilogue's last tile.
      const int ncells = (int)(P.lim - P.cell0);
      const int WC = A.win_cells;
      const float4* x4 = reinterpret_cast<const float4*>(A.master[A.cur & 1]);
      for (int job = ew * 32 + lane; job < ncells * (Cfg::C / 8); job += Cfg::EPI_WARPS * 32) {
        const int k = job / ncells, c = job - k * ncells;  // 8-channel chunk, cell of the group
        const long long gg = P.cell0 + c;
        const float4* src = x4 + (((gg >> 7) * (Cfg::C / 4) + 2 * k) << 7) + (gg & 127);
        const float4 a = src[0], b = src[128];
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        uint32_t h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          h[e] = pack_bf16(v[2 * e], v[2 * e + 1]);
          l[e] = pack_bf16(v[2 * e] - bf16lo_to_f32(h[e]), v[2 * e + 1] - bf16hi_to_f32(h[e]));
        }
        *reinterpret_cast<uint4*>(smem + L.win + (k * (WC + 1) + c) * 16) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(smem + L.rlo + (k * WC + c) * 16) = make_uint4(l[0], l[1], l[2], l[3]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[BAR_RES_LOADED]);
      // E2 reads cells that other epilogue warps loaded: wait for (acquire) the whole load
      if (!warp_wait(&bars[BAR_RES_LOADED], (uint32_t)ps & 1, fs, W_RES)) ok = false;
    }
    for (int s = 0; ok && s < A.n_steps; ++s) {
      const int in = (A.cur + s) & 1;
      const int out = in ^ 1;
      const float* xin = A.master[in];
      float* xout = A.master[out];
      uint16_t* mout = A.mirror[out];
      for (long long t = P.t0; t < P.t1;
           t += P.dt, ++it, wstage = (wstage + 1 == A.stages ? 0 : wstage + 1)) {
        const int slot = (int)(it % Cfg::NZ);
        const uint32_t zbase = tmem + lane_addr + slot * Cfg::SLOT_COLS;
        const int rg = (int)(it % Cfg::NACC);             // accumulator region of the tile
        const uint32_t ua = (uint32_t)(it / Cfg::NACC) & 1;  // its phase
        const uint32_t abase = tmem + lane_addr + Cfg::ACC_COL + rg * Cfg::HD;
        // ---- before E1: index math; the fire and given flags come from the stencil warps
        // (s_flags).
        const unsigned g = (unsigned)(P.cell0 + t * kTileM) + m;
        const bool valid = (long long)g < P.lim;
        int inst = 0;
        if (valid) inst = (int)fdiv(g, A.div_hw);
        constexpr int NQ = CH / 4;  // float4 chunks of this thread
        const float4* xin4 = reinterpret_cast<const float4*>(xin) + ((t * (Cfg::C / 4) + part * NQ) << 7) + m;
        // The part of the old state that E2 reads from global memory (the lo parts in the hi/lo
        // layout, else the fp32 state) is requested now, so that its latency overlaps E1.
        float4 xo[NQ];
        uint4 lo_pre[Cfg::HILO ? CH / 8 : 1];
        if constexpr (Cfg::HILO) {
          const uint4* lo4 = reinterpret_cast<const uint4*>(xin) + ((t * (Cfg::C / 8) + part * (CH / 8)) << 7) + m;
#pragma unroll
          for (int j = 0; j < CH / 8; ++j) lo_pre[j] = valid ? ld_nc_u4(lo4 + (j << 7)) : make_uint4(0u, 0u, 0u, 0u);
        } else if constexpr (!Cfg::RESIDENT) {
#pragma unroll
          for (int q = 0; q < NQ; ++q) xo[q] = valid ? ld_nc_f4(xin4 + (q << 7)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        // ---- E1: hidden = relu(acc1 + b1) -> bf16 (bf16 mode: over the accumulator columns of
        // the half already read, h of the half at [hh * HD / 2, hh * HD / 2 + HD / 4); split mode:
        // hi and lo parts into the consumed z slot)
        if (!warp_wait(&bars[(hh == 0 ? BAR_ACC_FULL : BAR_ACC_FULL_B) + rg], ua, fs, W_E1_ACC)) { ok = false; break; }
        tc_fence_after();
        if constexpr (!Cfg::SPLIT) {
          // bf16 mode: 16-column chunks, the next chunk's tensor-memory load in flight while this
          // one is converted (tcgen05.wait::ld waits for all of the thread's loads, so one load
          // is outstanding at a time)
          constexpr int NCHK = HPART / 16;
          uint32_t r0[16], r1[16];
          tmem_ld16(abase + part * HPART, r0);
#pragma unroll
          for (int c = 0; c < NCHK; ++c) {
            uint32_t(&rc)[16] = (c & 1) ? r1 : r0;
            uint32_t(&rn)[16] = (c & 1) ? r0 : r1;
            tc_wait_ld_regs(rc);
            if (c + 1 < NCHK) tmem_ld16(abase + part * HPART + (c + 1) * 16, rn);
            if (Cfg::PARTS_PER_HALF > 1 && sub == 0 && c == NCHK - 1) {
              // every column of this part is read: the second part of the half may overwrite them
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_relaxed(pair_bar);
            }
            const float4* bb = reinterpret_cast<const float4*>(s_b1 + part * HPART + c * 16);
            uint32_t hi[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 b = bb[q];
              const float2 h0 = __fadd2_rn(f2(__uint_as_float(rc[4 * q]), __uint_as_float(rc[4 * q + 1])), f2(b.x, b.y));
              const float2 h1 = __fadd2_rn(f2(__uint_as_float(rc[4 * q + 2]), __uint_as_float(rc[4 * q + 3])), f2(b.z, b.w));
              hi[2 * q] = pack_bf16_relu(h0.x, h0.y);
              hi[2 * q + 1] = pack_bf16_relu(h1.x, h1.y);
            }
            if (Cfg::PARTS_PER_HALF > 1 && sub > 0 && c == 0) {
              if (!warp_wait(pair_bar, (uint32_t)it & 1, fs, W_E1_PAIR)) { ok = false; break; }
              tc_fence_after();
            }
            tmem_st8(abase + hh * (Cfg::HD / 2) + (sub * HPART + c * 16) / 2, hi);
          }
        } else {
#pragma unroll 1
        for (int cbk = 0; cbk < HPART; cbk += E1C) {
          const int col = part * HPART + cbk;
          uint32_t r[E1C];
          if constexpr (E1C == 32) tmem_ld32(abase + col, *reinterpret_cast<uint32_t(*)[32]>(r));
          else tmem_ld16(abase + col, *reinterpret_cast<uint32_t(*)[16]>(r));
          tc_wait_ld_regs(r);
          uint32_t hi[E1C / 2];
          uint32_t lo[E1C / 2];
#pragma unroll
          for (int q = 0; q < E1C / 2; ++q) {
            const float h0 = fmaxf(__uint_as_float(r[2 * q]) + s_b1[col + 2 * q], 0.f);
            const float h1 = fmaxf(__uint_as_float(r[2 * q + 1]) + s_b1[col + 2 * q + 1], 0.f);
            hi[q] = pack_bf16(h0, h1);
            lo[q] = pack_bf16(h0 - bf16lo_to_f32(hi[q]), h1 - bf16hi_to_f32(hi[q]));
          }
          if constexpr (E1C == 32) {
            tmem_st16(zbase + col / 2, *reinterpret_cast<uint32_t(*)[16]>(hi));
            tmem_st16(zbase + Cfg::HD / 2 + col / 2, *reinterpret_cast<uint32_t(*)[16]>(lo));
          } else {
            tmem_st8(zbase + col / 2, *reinterpret_cast<uint32_t(*)[8]>(hi));
            tmem_st8(zbase + Cfg::HD / 2 + col / 2, *reinterpret_cast<uint32_t(*)[8]>(lo));
          }
        }
        }
        if (!ok) break;
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_relaxed(&bars[(hh == 0 ? BAR_H_FULL : BAR_H_FULL_B) + rg]);

        // ---- E2: dx = acc2 + b2; x' = x + f * dx; clamp; store.
        const int cl = (int)(t * kTileM) + m;  // resident: the cell's index in its group
        if constexpr (Cfg::RESIDENT) {
          // old state = hi (buffer s & 1) + lo of this thread's channels, in shared memory
          const int WC = A.win_cells;
#pragma unroll
          for (int j = 0; j < CH / 8; ++j) {
            const int k = part * (CH / 8) + j;
            uint4 hi = make_uint4(0u, 0u, 0u, 0u), lo = make_uint4(0u, 0u, 0u, 0u);
            if (valid) {
              hi = *reinterpret_cast<const uint4*>(smem + L.win + ((s & 1) * (WC + 1) * Cfg::NCH + k * (WC + 1) + cl) * 16);
              lo = *reinterpret_cast<const uint4*>(smem + L.rlo + (k * WC + cl) * 16);
            }
            xo[2 * j] = make_float4(bf16lo_to_f32(hi.x) + bf16lo_to_f32(lo.x), bf16hi_to_f32(hi.x) + bf16hi_to_f32(lo.x),
                                    bf16lo_to_f32(hi.y) + bf16lo_to_f32(lo.y), bf16hi_to_f32(hi.y) + bf16hi_to_f32(lo.y));
            xo[2 * j + 1] = make_float4(bf16lo_to_f32(hi.z) + bf16lo_to_f32(lo.z), bf16hi_to_f32(hi.z) + bf16hi_to_f32(lo.z),
                                        bf16lo_to_f32(hi.w) + bf16lo_to_f32(lo.w), bf16hi_to_f32(hi.w) + bf16hi_to_f32(lo.w));
          }
        } else if constexpr (Cfg::HILO) {
          // old state = hi, this tile's own cells in the window stage of the stencil, + lo
          const uint8_t* wst = smem + L.win + wstage * (A.win_cells + 1) * Cfg::ROWB;
#pragma unroll
          for (int j = 0; j < CH / 8; ++j) {
            const uint4 lo = lo_pre[j];
            const uint4 hi = *reinterpret_cast<const uint4*>(
                wst + ((part * (CH / 8) + j) * (A.win_cells + 1) + (m + W + 1)) * 16);
            xo[2 * j] = make_float4(bf16lo_to_f32(hi.x) + bf16lo_to_f32(lo.x), bf16hi_to_f32(hi.x) + bf16hi_to_f32(lo.x),
                                    bf16lo_to_f32(hi.y) + bf16lo_to_f32(lo.y), bf16hi_to_f32(hi.y) + bf16hi_to_f32(lo.y));
            xo[2 * j + 1] = make_float4(bf16lo_to_f32(hi.z) + bf16lo_to_f32(lo.z), bf16hi_to_f32(hi.z) + bf16hi_to_f32(lo.z),
                                        bf16lo_to_f32(hi.w) + bf16lo_to_f32(lo.w), bf16hi_to_f32(hi.w) + bf16hi_to_f32(lo.w));
          }
          // The stencil warps finished every read of this window before handing z to the MMA
          // warp, and this warp has used its hi values (the empty asm below takes the sums as
          // inputs, so the instructions that consume the shared-memory loads come before it):
          // release the stage to the loader.  The arrive is relaxed: a release arrive would first
          // wait for this thread's global stores of the previous tile.
#pragma unroll
          for (int q = 0; q < NQ; ++q) asm volatile("" ::"f"(xo[q].x), "f"(xo[q].y), "f"(xo[q].z), "f"(xo[q].w));
          __syncwarp();
          if (lane == 0) mbar_arrive_relaxed(&bars[BAR_WIN_EMPTY + wstage]);
        }
        if (!warp_wait(&bars[BAR_FLAGS + (it & 3)], (uint32_t)(it >> 2) & 1, fs, W_E2_FLAGS)) { ok = false; break; }

        const uint32_t fl = s_flags[(it & 3) * kTileM + m];
        const bool gv = (fl & 2u) != 0;
        const float f = (fl & 1u) ? 1.f : 0.f;
        if (!warp_wait(&bars[BAR_ACC2_FULL + rg], ua, fs, W_E2_ACC2)) { ok = false; break; }
        tc_fence_after();
        uint32_t r[CH];
        if constexpr (CH == 32) {
          tmem_ld32(abase + (Cfg::ACC2_COL - Cfg::ACC_COL) + part * CH, r);
        } else if constexpr (CH == 16) {
          tmem_ld16(abase + (Cfg::ACC2_COL - Cfg::ACC_COL) + part * CH, *reinterpret_cast<uint32_t(*)[16]>(r));
        } else {
          static_assert(CH == 8, "channels per epilogue thread");
          tmem_ld8(abase + (Cfg::ACC2_COL - Cfg::ACC_COL) + part * CH, *reinterpret_cast<uint32_t(*)[8]>(r));
        }
        tc_wait_ld_regs(r);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_relaxed(&bars[BAR_ACC_EMPTY + rg]);
        if (valid) {
          const float4* bb = reinterpret_cast<const float4*>(s_b2 + part * CH);
          const float2 ff = f2(f, f);
          float4* xout4 = reinterpret_cast<float4*>(xout) + ((t * (Cfg::C / 4) + part * NQ) << 7) + m;
          // Clamp (src/nca/model.py:430-438) of the input slice of given cells.  The state this
          // kernel reads is clamped already (the initial state is, every step keeps it so, and
          // the host follows the first step on an unclamped state with a clamp pass), so the old
          // values of those channels are kept: a select per channel, no branch, no reads of the
          // clamp rows.
          const int lo_c = A.in_off - part * CH;  // input slice relative to this thread's channels
          const unsigned long long slice = A.c_in >= 64 ? ~0ull : ((1ull << A.c_in) - 1ull);
          const uint32_t keep = (gv && lo_c < CH && lo_c + A.c_in > 0)
                                    ? (uint32_t)((slice << (lo_c + 32)) >> 32)
                                    : 0u;
          // the bf16 mirror of each 8 channels is stored as soon as they are done (fewer live
          // registers than packing all of them first)
          uint4* mout4 = reinterpret_cast<uint4*>(mout) + ((t * (Cfg::C / 8) + part * (CH / 8)) << 7) + m;
          uint4* lout4 = reinterpret_cast<uint4*>(xout) + ((t * (Cfg::C / 8) + part * (CH / 8)) << 7) + m;
          uint32_t pk[4], pl[4];
          // Test-time noise (src/nca/perturb.py:23-40): added after the update, before the clamp
          // (src/nca/model.py:544-546); only the NOISE instantiation carries this code.
          bool nz = false;
          int p_cell = 0;
          long long nid = 0;
          if constexpr (Cfg::NOISE) {
            p_cell = (int)(g - (unsigned)inst * A.HW);
            nid = A.inst_offset + (A.inst_id ? A.inst_id[inst] : inst);
            const long long step = A.step0 + s;
            if (A.noise_mode == 1) {
              nz = step < A.noise_until &&
                   u24(philox_tagged(A.seed, 1u, nid, 0u, step).x) < A.noise_p_t &&
                   u24(philox_tagged(A.seed, 2u, nid, (uint32_t)p_cell, step).x) < A.noise_p_s;
            } else if (A.noise_mode == 2) {
              nz = true;
            }
          }
#pragma unroll
          for (int q = 0; q < NQ; ++q) {
            const float4 b = bb[q];
            const float2 d0 = __fadd2_rn(f2(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1])), f2(b.x, b.y));
            const float2 d1 = __fadd2_rn(f2(__uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3])), f2(b.z, b.w));
            float2 y0 = __ffma2_rn(ff, d0, f2(xo[q].x, xo[q].y));
            float2 y1 = __ffma2_rn(ff, d1, f2(xo[q].z, xo[q].w));
            if constexpr (Cfg::NOISE) {
              if (nz) {
                float4 e;
                const int c0 = part * CH + 4 * q;  // first channel of this chunk
                if (A.noise_mode == 1) {
                  const float4 z = normal4(philox_tagged(A.seed, 3u, nid, (uint32_t)(p_cell * (Cfg::C / 4) + (c0 >> 2)),
                                                         A.step0 + s));
                  e = make_float4(A.noise_sigma * z.x, A.noise_sigma * z.y, A.noise_sigma * z.z,
                                  A.noise_sigma * z.w);
                } else {
                  const float* nb = A.noise + ((long long)inst * Cfg::C + c0) * A.HW + p_cell;
                  e = make_float4(nb[0], nb[A.HW], nb[2 * A.HW], nb[3 * A.HW]);
                }
                y0.x += e.x;
                y0.y += e.y;
                y1.x += e.z;
                y1.y += e.w;
              }
            }
            y0.x = (keep >> (4 * q + 0)) & 1u ? xo[q].x : y0.x;
            y0.y = (keep >> (4 * q + 1)) & 1u ? xo[q].y : y0.y;
            y1.x = (keep >> (4 * q + 2)) & 1u ? xo[q].z : y1.x;
            y1.y = (keep >> (4 * q + 3)) & 1u ? xo[q].w : y1.y;
            if constexpr (Cfg::RESIDENT) {
              if (s + 1 < A.n_steps) {
                // hi to the other buffer (the stencil's source at the next step), lo in place
                const uint32_t h0 = pack_bf16(y0.x, y0.y), h1 = pack_bf16(y1.x, y1.y);
                pk[2 * (q & 1)] = h0;
                pk[2 * (q & 1) + 1] = h1;
                pl[2 * (q & 1)] = pack_bf16(y0.x - bf16lo_to_f32(h0), y0.y - bf16hi_to_f32(h0));
                pl[2 * (q & 1) + 1] = pack_bf16(y1.x - bf16lo_to_f32(h1), y1.y - bf16hi_to_f32(h1));
                if (q & 1) {
                  const int k = part * (CH / 8) + (q >> 1);
                  const int WC = A.win_cells;
                  *reinterpret_cast<uint4*>(smem + L.win + (((s + 1) & 1) * (WC + 1) * Cfg::NCH + k * (WC + 1) + cl) * 16) =
                      make_uint4(pk[0], pk[1], pk[2], pk[3]);
                  *reinterpret_cast<uint4*>(smem + L.rlo + (k * WC + cl) * 16) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
                }
              } else {
                // the group's last step: the fp32 state and its bf16 copy to global memory
                const long long gt = (long long)(g >> 7), gr = g & 127;
                reinterpret_cast<float4*>(xout)[((gt * (Cfg::C / 4) + part * NQ + q) << 7) + gr] =
                    make_float4(y0.x, y0.y, y1.x, y1.y);
                pk[2 * (q & 1)] = pack_bf16(y0.x, y0.y);
                pk[2 * (q & 1) + 1] = pack_bf16(y1.x, y1.y);
                if (q & 1)
                  reinterpret_cast<uint4*>(mout)[((gt * (Cfg::C / 8) + part * (CH / 8) + (q >> 1)) << 7) + gr] =
                      make_uint4(pk[0], pk[1], pk[2], pk[3]);
              }
            } else if constexpr (Cfg::HILO) {
              // hi = bf16(y) to the mirror, lo = bf16(y - hi) to the low array
              const uint32_t h0 = pack_bf16(y0.x, y0.y), h1 = pack_bf16(y1.x, y1.y);
              pk[2 * (q & 1)] = h0;
              pk[2 * (q & 1) + 1] = h1;
              pl[2 * (q & 1)] = pack_bf16(y0.x - bf16lo_to_f32(h0), y0.y - bf16hi_to_f32(h0));
              pl[2 * (q & 1) + 1] = pack_bf16(y1.x - bf16lo_to_f32(h1), y1.y - bf16hi_to_f32(h1));
              if (q & 1) {
                mout4[(q >> 1) << 7] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                lout4[(q >> 1) << 7] = make_uint4(pl[0], pl[1], pl[2], pl[3]);
              }
            } else {
              xout4[q << 7] = make_float4(y0.x, y0.y, y1.x, y1.y);
              if constexpr (Cfg::SRC_BF16) {  // the stencil's bf16 copy
                pk[2 * (q & 1)] = pack_bf16(y0.x, y0.y);
                pk[2 * (q & 1) + 1] = pack_bf16(y1.x, y1.y);
                if (q & 1) mout4[(q >> 1) << 7] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              }
            }
          }
        }
        if ((Cfg::RESIDENT || Cfg::TILEDEP) && part == 0 && A.updates != nullptr) {
          // fired cells per instance (the grid-barrier streaming form counts in the stencil)
          const bool fired = valid && f > 0.f;
          const unsigned grp = __match_any_sync(0xffffffffu, valid ? inst : -1);
          const unsigned fm = __ballot_sync(0xffffffffu, fired);
          if (valid && lane == __ffs(grp) - 1) {
            const int cnt = __popc(fm & grp);
            if (cnt) atomicAdd(&A.updates[inst], (unsigned)cnt);
          }
        }
        if constexpr (Cfg::RESIDENT || Cfg::ADAPTIVE) {
          // this warp is done with the tile (its stores are ordered before the release): the
          // resident stencil's wait for the next step, or the confidence warps, read it
          __syncwarp();
          if (lane == 0)
            asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(s_prog + ew)), "r"(it + 1u) : "memory");
        }
        if constexpr (Cfg::TILEDEP) {
          // this warp's stores of the tile are issued: count it for the publisher lane (the warp
          // barrier orders the lanes' stores before lane 0's release)
          __syncwarp();
          if (lane == 0) asm volatile("red.release.cta.shared::cta.add.u32 [%0], 1;" ::"r"(smem_u32(s_tiles_done)) : "memory");
        }
      }
      if constexpr (!Cfg::TILEDEP && !Cfg::RESIDENT) {
        // Step done: this CTA's stores of step s are complete.  The barrier also ORs the failure
        // flags of the epilogue warps so that they leave the step loop together.
        unsigned any_fail;
        asm volatile(
            "{\n\t.reg .pred p, q;\n\t"
            "setp.ne.u32 p, %1, 0;\n\t"
            "bar.red.or.pred q, 1, %2, p;\n\t"
            "selp.u32 %0, 1, 0, q;\n\t}"
            : "=r"(any_fail)
            : "r"((unsigned)(!ok || *(volatile int*)abort_flag != 0)),
              "n"(Cfg::EPI_WARPS * 32 + (Cfg::ADAPTIVE ? 64 : 0))
            : "memory");
        if (any_fail) { ok = false; break; }
        if (threadIdx.x == kEpiWarp0 * 32) {
          __threadfence();
          atomicAdd(reinterpret_cast<unsigned*>(&A.ctrl[2]), 1u);
        }
      }
    }
    if constexpr (Cfg::RESIDENT) {
      // End of a group: every epilogue warp is done with it (the next group's load overwrites
      // its state).  The barrier also ORs the warps' failure flags so that they leave together.
      unsigned any_fail;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\t"
          "setp.ne.u32 p, %1, 0;\n\t"
          "bar.red.or.pred q, 2, %2, p;\n\t"
          "selp.u32 %0, 1, 0, q;\n\t}"
          : "=r"(any_fail)
          : "r"((unsigned)(!ok || *(volatile int*)abort_flag != 0)), "n"(Cfg::EPI_WARPS * 32)
          : "memory");
      if (any_fail) { ok = false; break; }
    }
    }  // passes
  }

  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

}  // namespace nca
