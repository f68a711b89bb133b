// api.cu -- C ABI of libnca_b200 (declared in include/nca_b200.h): host entry points, the step
// kernel instantiations and the small kernels around it (state layout conversion, readout,
// conf@K selection, niche-capped pruning with refill, state cloning).
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <atomic>

#include "../../include/nca_b200.h"
#include "launch.cuh"
#include "step_kernel.cuh"

using namespace nca;

namespace {

inline int32_t cuda_status(cudaError_t e) { return e == cudaSuccess ? NCA_OK : NCA_ERR_CUDA; }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline long long n_tiles_of(long long cells) { return (cells + kTileM - 1) / kTileM; }

inline size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// ------------------------------------------------------------------------------ bf16 (host)
inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return (uint16_t)(u >> 16);
}

// Writes a (rows x K) row-major fp32 matrix as the K-major, 128B-swizzled bf16 image that a
// tcgen05 shared-memory descriptor with SWIZZLE_128B reads: K in blocks of 64, each block
// [rows][128 B], 16-byte chunk c of row r stored at chunk position c ^ (r & 7).
void pack_sw128(const float* w, int rows, int K, uint16_t* out) {
  const int kb_n = K / 64;
  for (int kb = 0; kb < kb_n; ++kb)
    for (int r = 0; r < rows; ++r)
      for (int c = 0; c < 8; ++c)
        for (int e = 0; e < 8; ++e) {
          const int k = kb * 64 + c * 8 + e;
          const size_t dst = (size_t)kb * rows * 64 + (size_t)r * 64 + ((c ^ (r & 7)) * 8) + e;
          out[dst] = f32_to_bf16_rne(w[(size_t)r * K + k]);
        }
}

// ------------------------------------------------------------------------- state kernels
__device__ __forceinline__ float clamp_value(const NcaBatchDesc& b, int c_in, int in_off, int inst,
                                             int p, int c, float v) {
  const int row = b.inst_row ? b.inst_row[inst] : inst / b.trials;
  const int ci = c - in_off;
  if (ci >= 0 && ci < c_in && b.given[(long long)row * b.height * b.width + p])
    return b.clamp[((long long)row * b.height * b.width + p) * c_in + ci];
  return v;
}

// Copies 16-byte unit u of the state of cell gs to cell gd: hi and lo bf16 units (C/8 units) in
// the hi/lo layout, else fp32 master units (C/4) and, for even u, the bf16 mirror's unit u/2.
__device__ __forceinline__ void copy_cell_unit(const float* smaster, const uint16_t* smirror,
                                               float* dmaster, uint16_t* dmirror, int C, long long gs,
                                               long long gd, int u) {
  if (smirror && hilo_layout(C, true)) {
    const int C8 = C / 8;
    const long long os = (((gs >> 7) * C8 + u) << 7) + (gs & 127);
    const long long od = (((gd >> 7) * C8 + u) << 7) + (gd & 127);
    reinterpret_cast<uint4*>(dmirror)[od] = reinterpret_cast<const uint4*>(smirror)[os];
    reinterpret_cast<uint4*>(dmaster)[od] = reinterpret_cast<const uint4*>(smaster)[os];
    return;
  }
  const int C4 = C / 4;
  const long long os = (((gs >> 7) * C4 + u) << 7) + (gs & 127);
  const long long od = (((gd >> 7) * C4 + u) << 7) + (gd & 127);
  reinterpret_cast<float4*>(dmaster)[od] = reinterpret_cast<const float4*>(smaster)[os];
  if (smirror && (u & 1) == 0) {
    const int C8 = C / 8;
    const long long ms = (((gs >> 7) * C8 + (u >> 1)) << 7) + (gs & 127);
    const long long md = (((gd >> 7) * C8 + (u >> 1)) << 7) + (gd & 127);
    reinterpret_cast<uint4*>(dmirror)[md] = reinterpret_cast<const uint4*>(smirror)[ms];
  }
}

// The clamp of src/nca/model.py:430-438 on the current state: one thread per cell writes the
// clamp values over the input slice of the given cells (fp32 state and bf16 mirror).  Run after
// the first step on a state that was not clamped (loaded from outside the library); the step
// kernel itself keeps the slice of given cells as it finds it.
__global__ void clamp_fix_kernel(float* master, uint16_t* mirror, int C, long long total, int hw,
                                 NcaBatchDesc b, int c_in, int in_off) {
  const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= total) return;
  const int inst = (int)(g / hw);
  const int p = (int)(g - (long long)inst * hw);
  const int row = b.inst_row ? b.inst_row[inst] : inst / b.trials;
  if (!b.given[(long long)row * hw + p]) return;
  for (int ci = 0; ci < c_in; ++ci)
    state_put(master, mirror, C, g, in_off + ci, b.clamp[((long long)row * hw + p) * c_in + ci]);
}

// Damage (src/nca/rollout.py:206-212): one thread per cell; a masked cell gets a zero state, and
// a given cell its clamp values again.
__global__ void damage_kernel(float* master, uint16_t* mirror, int C, long long total, int hw,
                              NcaBatchDesc b, int c_in, int in_off, const uint8_t* masks) {
  const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= total) return;
  const int inst = (int)(g / hw);
  const int p = (int)(g - (long long)inst * hw);
  const int row = b.inst_row ? b.inst_row[inst] : inst / b.trials;
  if (!masks[(long long)row * hw + p]) return;
  const bool gv = b.given[(long long)row * hw + p] != 0;
  for (int c = 0; c < C; ++c) {
    const int ci = c - in_off;
    const float v = (gv && ci >= 0 && ci < c_in) ? b.clamp[((long long)row * hw + p) * c_in + ci] : 0.f;
    state_put(master, mirror, C, g, c, v);
  }
}

// One thread per (tile, 8-channel group, row): writes 8 channels of one cell.
// mode 0: zero state + clamp; mode 1: load from NCHW.
__global__ void state_fill_kernel(float* master, uint16_t* mirror, int C, long long n_tiles,
                                  long long total, int hw, NcaBatchDesc b, int c_in, int in_off,
                                  const float* x_nchw, int mode) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int C8 = C / 8;
  if (idx >= n_tiles * C8 * kTileM) return;
  const int m = (int)(idx & 127);
  const long long rest = idx >> 7;
  const int c8 = (int)(rest % C8);
  const long long t = rest / C8;
  const long long g = t * kTileM + m;
  float v[8];
  for (int e = 0; e < 8; ++e) v[e] = 0.f;
  if (g < total) {
    const int inst = (int)(g / hw);
    const int p = (int)(g - (long long)inst * hw);
    for (int e = 0; e < 8; ++e) {
      const int c = c8 * 8 + e;
      float x = 0.f;
      if (mode == 1) x = x_nchw[((long long)inst * C + c) * hw + p];
      else x = clamp_value(b, c_in, in_off, inst, p, c, 0.f);
      v[e] = x;
    }
  }
  if (mirror && hilo_layout(C, true)) {  // hi and lo parts
    uint32_t h[4], l[4];
    for (int e = 0; e < 4; ++e) {
      h[e] = pack_bf16(v[2 * e], v[2 * e + 1]);
      l[e] = pack_bf16(v[2 * e] - bf16lo_to_f32(h[e]), v[2 * e + 1] - bf16hi_to_f32(h[e]));
    }
    const long long o = ((t * (C / 8) + c8) * kTileM + m) * 8;
    *reinterpret_cast<uint4*>(mirror + o) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(master) + o) = make_uint4(l[0], l[1], l[2], l[3]);
  } else {
    for (int hq = 0; hq < 2; ++hq) {
      const int c4 = c8 * 2 + hq;
      *reinterpret_cast<float4*>(master + ((t * (C / 4) + c4) * kTileM + m) * 4) =
          make_float4(v[hq * 4 + 0], v[hq * 4 + 1], v[hq * 4 + 2], v[hq * 4 + 3]);
    }
    if (mirror) {
      const uint4 pk = make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]),
                                  pack_bf16(v[6], v[7]));
      *reinterpret_cast<uint4*>(mirror + ((t * (C / 8) + c8) * kTileM + m) * 8) = pk;
    }
  }
}

__global__ void state_store_kernel(const float* master, const uint16_t* mirror, int C,
                                   long long total, int hw, float* x_nchw) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total * C) return;
  // idx enumerates NCHW order: ((inst * C + c) * hw + p)
  const int p = (int)(idx % hw);
  const long long r = idx / hw;
  const int c = (int)(r % C);
  const long long inst = r / C;
  x_nchw[idx] = state_get(master, mirror, C, inst * hw + p, c);
}

// ------------------------------------------------------------------------------- readout
struct ReadoutArgs {
  int C, hw, n_inst, c_out, out_off, n_out, head_kind;
  float head_w[16][16];
  float head_b[16];
  int out_tokens[16];
};

// One block per instance.  head_readout of every cell (argmax as torch.argmax, the head's
// confidence clamped to [0, 1], src/nca/model.py:596-633), the decoded token (given cells show
// their input, src/nca/rollout.py:74-82), the board confidence and, with targets, the accuracy.
__global__ void readout_kernel(const float* master, const uint16_t* mirror, NcaBatchDesc b, ReadoutArgs R, uint8_t* pred,
                               float* cell_conf, float* board_conf, const uint8_t* targets,
                               float* cell_acc, uint8_t* exact) {
  const int inst = blockIdx.x;
  const int row = b.inst_row ? b.inst_row[inst] : inst / b.trials;
  float conf_sum = 0.f, correct = 0.f, n_mut = 0.f;
  for (int p = threadIdx.x; p < R.hw; p += blockDim.x) {
    const long long g = (long long)inst * R.hw + p;
    float xo[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      xo[c] = 0.f;
      if (c < R.c_out) xo[c] = state_get(master, mirror, R.C, g, R.out_off + c);
    }
    float conf;
    int arg;
    head_readout(R.head_kind, R.n_out, R.c_out, R.head_w, R.head_b, xo, conf, arg);
    conf_sum += conf;
  const long long bp = (long long)row * R.hw + p;
    const bool gv = b.given[bp] != 0;
    const int tok = gv ? (int)b.inputs[bp] : R.out_tokens[arg];
    if (pred) pred[(long long)inst * R.hw + p] = (uint8_t)tok;
    if (cell_conf) cell_conf[(long long)inst * R.hw + p] = conf;
    if (targets && !gv) {
      n_mut += 1.f;
      correct += (tok == (int)targets[bp]) ? 1.f : 0.f;
    }
  }
  __shared__ float red[3][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int o = 16; o; o >>= 1) {
    conf_sum += __shfl_xor_sync(0xffffffffu, conf_sum, o);
    correct += __shfl_xor_sync(0xffffffffu, correct, o);
    n_mut += __shfl_xor_sync(0xffffffffu, n_mut, o);
  }
  if (lane == 0) { red[0][w] = conf_sum; red[1][w] = correct; red[2][w] = n_mut; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f, c = 0.f, n = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) { a += red[0][i]; c += red[1][i]; n += red[2][i]; }
    if (board_conf) board_conf[inst] = a / (float)R.hw;
    if (targets) {
      const float nm = fmaxf(n, 1.f);
      if (cell_acc) cell_acc[inst] = c / nm;
      if (exact) exact[inst] = (c == nm) ? 1 : 0;
    }
  }
}

// Fire probability of every cell of the current state under the confidence rules (the values
// the step kernel's epilogue then keeps up to date): head_readout of the cell's readout slice,
// then the continuous or the threshold rule (src/nca/model.py:566-593).  One thread per cell of
// the tiled layout; rows past the last cell get 0.
__global__ void fire_p_kernel(const float* master, const uint16_t* mirror, int C, long long n_cells,
                              long long total, int hw, NcaBatchDesc b, ReadoutArgs R, int mode,
                              float scale, float bias, float p_low, float tau, float p_fire,
                              int given_confident, float* fire_p) {
  const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n_cells) return;
  if (g >= total) {
    fire_p[g] = 0.f;
    return;
  }
  const int inst = (int)(g / hw);
  const int p = (int)(g - (long long)inst * hw);
  const int row = b.inst_row ? b.inst_row[inst] : inst / b.trials;
  float xo[16];
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    xo[c] = 0.f;
    if (c < R.c_out) xo[c] = state_get(master, mirror, C, g, R.out_off + c);
  }
  float conf;
  int arg;
  head_readout(R.head_kind, R.n_out, R.c_out, R.head_w, R.head_b, xo, conf, arg);
  fire_p[g] = adaptive_prob(mode, conf, b.given[(long long)row * hw + p] != 0, scale, bias, p_low, tau,
                            p_fire, given_confident);
}

// Order of np.argmax over (alive ? conf : -inf): a NaN is larger than every number (argmax
// returns the first NaN), ties go to the smaller index.
__device__ __forceinline__ bool select_better(float v, int k, float bv, int bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn || bn) return vn && (!bn || k < bi);
  return v > bv || (v == bv && k < bi);
}

// One warp per board: first index of the maximum of (alive ? conf : -inf) over k < k_limit,
// with the NaN rule of np.argmax (src/nca/rollout.py:331-332).
__global__ void select_kernel(const float* conf, const uint8_t* alive, int n_boards, int K,
                              int k_limit, int* best_idx, float* best_conf, const uint8_t* pred,
                              int hw, uint8_t* best_pred) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n_boards) return;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int k = lane; k < k_limit; k += 32) {
    const long long i = (long long)warp * K + k;
    const float v = (alive == nullptr || alive[i]) ? conf[i] : -INFINITY;
    if (select_better(v, k, bv, bi)) { bv = v; bi = k; }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (select_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if (bi == 0x7fffffff) bi = 0;
  if (lane == 0) {
    if (best_idx) best_idx[warp] = bi;
    if (best_conf) best_conf[warp] = bv;
  }
  if (pred && best_pred) {
    const uint8_t* src = pred + ((long long)warp * K + bi) * hw;
    for (int p = lane; p < hw; p += 32) best_pred[(long long)warp * hw + p] = src[p];
  }
}

// FNV-1a 64-bit over the decoded grid (Fowler, Noll, Vo; public-domain hash).
__device__ __forceinline__ uint64_t fnv1a64(const uint8_t* p, int n) {
  uint64_t h = 1469598103934665603ull;
  for (int i = 0; i < n; ++i) { h ^= p[i]; h *= 1099511628211ull; }
  return h;
}

// One block of K threads per board.
__global__ void prune_refill_kernel(const uint8_t* pred, const float* conf, int K, int hw,
                                    int n_cap, int* src, uint8_t* kept_out) {
  extern __shared__ uint8_t sm[];
  uint64_t* hsh = reinterpret_cast<uint64_t*>(sm);
  float* cf = reinterpret_cast<float*>(hsh + K);
  int* niche = reinterpret_cast<int*>(cf + K);
  int* kept = niche + K;
  int* by_rank = kept + K;
  const int board = blockIdx.x;
  const int k = threadIdx.x;
  const uint8_t* base = pred + (long long)board * K * hw;
  if (k < K) {
    hsh[k] = fnv1a64(base + (long long)k * hw, hw);
    cf[k] = conf[(long long)board * K + k];
  }
  __syncthreads();
  if (k < K) {
    int nid = k;
    for (int j = 0; j < k; ++j) {
      if (hsh[j] != hsh[k]) continue;
      const uint8_t* a = base + (long long)j * hw;
      const uint8_t* b = base + (long long)k * hw;
      bool eq = true;
      for (int p = 0; p < hw; ++p)
        if (a[p] != b[p]) { eq = false; break; }
      if (eq) { nid = j; break; }
    }
    niche[k] = nid;
  }
  __syncthreads();
  if (k < K) {
    int rank = 0;
    for (int j = 0; j < K; ++j)
      if (niche[j] == niche[k] && (cf[j] > cf[k] || (cf[j] == cf[k] && j < k))) ++rank;
    kept[k] = rank < n_cap ? 1 : 0;
  }
  __syncthreads();
  int n_kept = 0;
  for (int j = 0; j < K; ++j) n_kept += kept[j];
  if (k < K && kept[k]) {
    int srank = 0;
    for (int j = 0; j < K; ++j)
      if (kept[j] && (cf[j] > cf[k] || (cf[j] == cf[k] && j < k))) ++srank;
    by_rank[srank] = k;
  }
  __syncthreads();
  if (k < K) {
    int s = k;
    if (!kept[k]) {
      int d = 0;
      for (int j = 0; j < k; ++j) d += kept[j] ? 0 : 1;
      s = by_rank[d % n_kept];
    }
    src[(long long)board * K + k] = board * K + s;
    if (kept_out) kept_out[(long long)board * K + k] = (uint8_t)kept[k];
  }
}

// Niches of the halving rule (src/nca/pruning.py:39-46), one block per board: the board's alive
// trials are the rows [row_start[b], row_start[b + 1]) (increasing trial order).  niche[r] is the
// index of r's niche in order of first appearance, rank[r] its position in the niche by
// decreasing confidence, ties by row (Python's stable sort on -conf).
__global__ void niche_kernel(const uint8_t* pred, const float* conf, const int* row_start, int hw,
                             int max_rows, int* niche, int* rank, int* n_niches) {
  extern __shared__ uint8_t sm[];
  const int b = blockIdx.x;
  const int r0 = row_start[b], nr = row_start[b + 1] - r0;
  if (nr < 0 || nr > max_rows) return;  // inconsistent row_start: leave the outputs untouched
  uint64_t* hsh = reinterpret_cast<uint64_t*>(sm);
  float* cf = reinterpret_cast<float*>(hsh + nr);
  int* first = reinterpret_cast<int*>(cf + nr);   // first row (local) with the same grid
  int* nid = first + nr;                          // niche index of the row
  for (int i = threadIdx.x; i < nr; i += blockDim.x) {
    hsh[i] = fnv1a64(pred + (long long)(r0 + i) * hw, hw);
    cf[i] = conf[r0 + i];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nr; i += blockDim.x) {
    int f = i;
    for (int j = 0; j < i; ++j) {
      if (hsh[j] != hsh[i]) continue;
      const uint8_t* a = pred + (long long)(r0 + j) * hw;
      const uint8_t* c = pred + (long long)(r0 + i) * hw;
      bool eq = true;
      for (int p = 0; p < hw; ++p)
        if (a[p] != c[p]) { eq = false; break; }
      if (eq) { f = j; break; }
    }
    first[i] = f;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nr; i += blockDim.x) {
    int idx = 0;  // niches that appear before this row's niche
    for (int j = 0; j < first[i]; ++j) idx += first[j] == j ? 1 : 0;
    nid[i] = idx;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nr; i += blockDim.x) {
    int rk = 0;
    for (int j = 0; j < nr; ++j)
      if (nid[j] == nid[i] && (cf[j] > cf[i] || (cf[j] == cf[i] && j < i))) ++rk;
    niche[r0 + i] = nid[i];
    rank[r0 + i] = rk;
  }
  if (threadIdx.x == 0) {
    int cnt = 0;
    for (int j = 0; j < nr; ++j) cnt += first[j] == j ? 1 : 0;
    n_niches[b] = cnt;
  }
}

// Survivors of the halving (src/nca/pruning.py:47-61), one block per board.  The member of rank d
// of niche j sits at position sum_j' min(len_j', d) + #{j' before j in the order: len_j' > d} of
// the round-robin sequence (len = niche size capped at n_cap); the first floor(alive / 2)
// positions survive.  Boards with at most one alive trial keep it.
__global__ void halving_kernel(const int* niche, const int* rank, const int* n_niches,
                               const int* row_start, const int* order, const int* order_start,
                               int n_cap, int max_rows, uint8_t* keep) {
  extern __shared__ int shm[];
  const int b = blockIdx.x;
  const int r0 = row_start[b], nr = row_start[b + 1] - r0;
  const int nn = n_niches[b];
  int* len = shm;         // capped niche sizes
  int* pos = shm + nr;    // position of each niche in the drawn order
  if (nr > max_rows || nn > nr) return;  // inconsistent arguments: leave keep untouched
  if (nr <= 1) {
    for (int i = threadIdx.x; i < nr; i += blockDim.x) keep[r0 + i] = 1;
    return;
  }
  for (int j = threadIdx.x; j < nn; j += blockDim.x) {
    len[j] = 0;
    const int o = order[order_start[b] + j];
    if (o >= 0 && o < nn) pos[o] = j;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nr; i += blockDim.x)
    if (rank[r0 + i] < n_cap) atomicAdd(&len[niche[r0 + i]], 1);
  __syncthreads();
  const int target = nr / 2;
  for (int i = threadIdx.x; i < nr; i += blockDim.x) {
    const int j = niche[r0 + i], d = rank[r0 + i];
    bool k = false;
    if (d < n_cap) {
      int p = 0;
      for (int q = 0; q < nn; ++q) {
        p += len[q] < d ? len[q] : d;
        if (pos[q] < pos[j] && len[q] > d) ++p;
      }
      k = p < target;
    }
    keep[r0 + i] = k ? 1 : 0;
  }
}

// One thread per (destination instance, cell, 16-byte unit): dst instance i <- src sel[i].
__global__ void gather_kernel(const float* smaster, const uint16_t* smirror, float* dmaster,
                              uint16_t* dmirror, int C, int hw, int n_dst, const int* sel) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int U = (smirror && hilo_layout(C, true)) ? C / 8 : C / 4;
  if (idx >= (long long)n_dst * hw * U) return;
  const int u = (int)(idx % U);
  const long long g = idx / U;
  const int i = (int)(g / hw);
  const int p = (int)(g - (long long)i * hw);
  copy_cell_unit(smaster, smirror, dmaster, dmirror, C, (long long)sel[i] * hw + p, g, u);
}

// One thread per (destination instance, cell, 16-byte unit of the state).
__global__ void clone_kernel(float* master, uint16_t* mirror, int C, int hw, int n_inst,
                             const int* src) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int U = (mirror && hilo_layout(C, true)) ? C / 8 : C / 4;
  if (idx >= (long long)n_inst * hw * U) return;
  const int u = (int)(idx % U);
  const long long cell = idx / U;
  const int inst = (int)(cell / hw);
  const int p = (int)(cell - (long long)inst * hw);
  const int s = src[inst];
  if (s == inst) return;
  copy_cell_unit(master, mirror, master, mirror, C, (long long)s * hw + p, (long long)inst * hw + p, u);
}

__global__ void selftest_wait_kernel(int* ctrl, unsigned long long timeout_ns) {
  __shared__ int abort_flag;
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  FailState fs;
  fs.ctrl = ctrl;
  fs.cta_abort = &abort_flag;
  fs.timeout_ns = timeout_ns;
  fs.deadline_ns = 0;
  // Nothing ever arrives on `bar`: the bounded wait must give up and report a timeout.
  if (threadIdx.x < 32) warp_wait(&bar, 0, fs, 99);
  __syncthreads();
}

bool model_ok(const NcaModelDesc* m) {
  if (!m || !m->weights || !m->b1 || !m->b2) return false;
  if (m->perception != 4 * m->channels) return false;
  if (m->c_in < 0 || m->in_offset < 0 || m->in_offset + m->c_in > m->channels) return false;
  if (m->c_out < 1 || m->c_out > NCA_B200_MAX_OUT || m->out_offset < 0 ||
      m->out_offset + m->c_out > m->channels)
    return false;
  if (m->n_out < 1 || m->n_out > NCA_B200_MAX_OUT) return false;
  if (m->head_kind != NCA_HEAD_LINEAR && m->head_kind != NCA_HEAD_L2) return false;
  if (m->channels > 64) return false;
  return true;
}

bool batch_ok(const NcaBatchDesc* b) {
  return b && b->n_inst > 0 && b->height > 0 && b->width > 0 && b->trials > 0 && b->given &&
         b->clamp;
}

}  // namespace

extern "C" {

int32_t nca_b200_abi_version(void) { return NCA_B200_ABI_VERSION; }

const char* nca_b200_status_string(int32_t s) {
  switch (s) {
    case NCA_OK: return "ok";
    case NCA_ERR_INVALID: return "invalid argument";
    case NCA_ERR_UNSUPPORTED: return "unsupported configuration";
    case NCA_ERR_CUDA: return "CUDA runtime error";
    case NCA_ERR_TIMEOUT: return "a bounded wait inside a kernel ran out";
    case NCA_ERR_DEVICE: return "no usable sm_100 device";
    case NCA_ERR_KERNEL: return "kernel-side check failed";
    case NCA_ERR_SCRATCH: return "request larger than the static scratch of nca_b200_run_steps_static";
    default: return "unknown status";
  }
}

int32_t nca_b200_device_info(int32_t device, int32_t* sm_count, int32_t* cc_major,
                             int32_t* cc_minor) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return NCA_ERR_DEVICE;
  int sms = 0, ma = 0, mi = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&ma, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&mi, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess)
    return NCA_ERR_CUDA;
  if (sm_count) *sm_count = sms;
  if (cc_major) *cc_major = ma;
  if (cc_minor) *cc_minor = mi;
  if (ma != 10) return NCA_ERR_DEVICE;
  cudaFuncAttributes fa;
  if (step_kernel_attributes(&fa) != cudaSuccess)
    return NCA_ERR_DEVICE;
  return NCA_OK;
}

int32_t nca_b200_weights_bytes(int32_t channels, int32_t perception, int32_t hidden,
                               size_t* bytes) {
  if (!bytes || channels <= 0 || perception <= 0 || hidden <= 0) return NCA_ERR_INVALID;
  if (perception % 64 || hidden % 64 || channels % 8) return NCA_ERR_UNSUPPORTED;
  *bytes = ((size_t)hidden * perception + (size_t)channels * hidden) * 2;
  return NCA_OK;
}

int32_t nca_b200_pack_weights(const float* w1, const float* w2, int32_t channels,
                              int32_t perception, int32_t hidden, void* image_host) {
  size_t bytes = 0;
  int32_t s = nca_b200_weights_bytes(channels, perception, hidden, &bytes);
  if (s != NCA_OK) return s;
  if (!w1 || !w2 || !image_host) return NCA_ERR_INVALID;
  uint16_t* out = reinterpret_cast<uint16_t*>(image_host);
  pack_sw128(w1, hidden, perception, out);
  pack_sw128(w2, channels, hidden, out + (size_t)hidden * perception);
  return NCA_OK;
}

int32_t nca_b200_state_bytes(int32_t n_inst, int32_t hw, int32_t channels, int32_t precision,
                             size_t* bytes) {
  if (!bytes || n_inst <= 0 || hw <= 0 || channels <= 0 || channels % 16) return NCA_ERR_INVALID;
  const long long tiles = n_tiles_of((long long)n_inst * hw);
  // fp32 master (+ bf16 mirror in bf16 mode), or hi (mirror) and lo (master) bf16 arrays
  const bool hl = hilo_layout(channels, precision == NCA_PREC_BF16);
  const size_t master = align256((size_t)tiles * kTileM * channels * (hl ? 2 : 4));
  const size_t mirror = precision == NCA_PREC_BF16 ? align256((size_t)tiles * kTileM * channels * 2) : 0;
  // + per-tile step counters + per-cell fire probabilities (confidence rules)
  *bytes = 2 * master + 2 * mirror + align256((size_t)tiles * 4) + align256((size_t)tiles * kTileM * 4);
  return NCA_OK;
}

int32_t nca_b200_state_bind(NcaState* st, void* buffer, size_t bytes, int32_t n_inst, int32_t hw,
                            int32_t channels, int32_t precision) {
  size_t need = 0;
  int32_t s = nca_b200_state_bytes(n_inst, hw, channels, precision, &need);
  if (s != NCA_OK) return s;
  if (!st || !buffer || bytes < need || (reinterpret_cast<uintptr_t>(buffer) & 255))
    return NCA_ERR_INVALID;
  if (precision != NCA_PREC_BF16 && precision != NCA_PREC_SPLIT) return NCA_ERR_INVALID;
  const long long tiles = n_tiles_of((long long)n_inst * hw);
  const bool hl = hilo_layout(channels, precision == NCA_PREC_BF16);
  const size_t master = align256((size_t)tiles * kTileM * channels * (hl ? 2 : 4));
  const size_t mirror = precision == NCA_PREC_BF16 ? align256((size_t)tiles * kTileM * channels * 2) : 0;
  uint8_t* p = reinterpret_cast<uint8_t*>(buffer);
  st->n_inst = n_inst;
  st->hw = hw;
  st->channels = channels;
  st->precision = precision;
  st->n_tiles = tiles;
  st->master[0] = reinterpret_cast<float*>(p);
  st->master[1] = reinterpret_cast<float*>(p + master);
  st->mirror[0] = mirror ? reinterpret_cast<uint16_t*>(p + 2 * master) : nullptr;
  st->mirror[1] = mirror ? reinterpret_cast<uint16_t*>(p + 2 * master + mirror) : nullptr;
  st->tile_steps = reinterpret_cast<uint32_t*>(p + 2 * master + 2 * mirror);
  st->fire_p = reinterpret_cast<float*>(p + 2 * master + 2 * mirror + align256((size_t)tiles * 4));
  st->cur = 0;
  st->clamped = 0;
  return NCA_OK;
}

int32_t nca_b200_state_init(NcaState* st, const NcaModelDesc* m, const NcaBatchDesc* b,
                            void* stream) {
  if (!st || !m || !batch_ok(b) || b->n_inst != st->n_inst || b->height * b->width != st->hw)
    return NCA_ERR_INVALID;
  const long long n = st->n_tiles * (st->channels / 8) * kTileM;
  const int bs = 256;
  state_fill_kernel<<<(unsigned)((n + bs - 1) / bs), bs, 0, as_stream(stream)>>>(
      st->master[st->cur], st->mirror[st->cur], st->channels, st->n_tiles,
      (long long)st->n_inst * st->hw, st->hw, *b, m->c_in, m->in_offset, nullptr, 0);
  st->clamped = 1;
  return cuda_status(cudaGetLastError());
}

int32_t nca_b200_state_load_nchw(NcaState* st, const float* x_nchw, void* stream) {
  if (!st || !x_nchw) return NCA_ERR_INVALID;
  NcaBatchDesc dummy;
  memset(&dummy, 0, sizeof(dummy));
  dummy.trials = 1;
  const long long n = st->n_tiles * (st->channels / 8) * kTileM;
  const int bs = 256;
  state_fill_kernel<<<(unsigned)((n + bs - 1) / bs), bs, 0, as_stream(stream)>>>(
      st->master[st->cur], st->mirror[st->cur], st->channels, st->n_tiles,
      (long long)st->n_inst * st->hw, st->hw, dummy, 0, 0, x_nchw, 1);
  st->clamped = 0;
  return cuda_status(cudaGetLastError());
}

int32_t nca_b200_state_store_nchw(const NcaState* st, float* x_nchw, void* stream) {
  if (!st || !x_nchw) return NCA_ERR_INVALID;
  const long long n = (long long)st->n_inst * st->hw * st->channels;
  const int bs = 256;
  state_store_kernel<<<(unsigned)((n + bs - 1) / bs), bs, 0, as_stream(stream)>>>(
      st->master[st->cur], st->mirror[st->cur], st->channels, (long long)st->n_inst * st->hw, st->hw,
      x_nchw);
  return cuda_status(cudaGetLastError());
}

int32_t nca_b200_run_steps(const NcaModelDesc* m, const NcaBatchDesc* b, NcaState* st,
                           int32_t n_steps, const NcaFireDesc* fire, int32_t* ctrl,
                           int32_t timeout_ms, void* stream) {
  if (!model_ok(m) || !batch_ok(b) || !st || !fire || !ctrl || n_steps < 0) return NCA_ERR_INVALID;
  if (b->n_inst != st->n_inst || b->height * b->width != st->hw || m->channels != st->channels)
    return NCA_ERR_INVALID;
  if (fire->mode == NCA_FIRE_MASK && !fire->masks) return NCA_ERR_INVALID;
  if ((fire->mode == NCA_FIRE_ADAPTIVE_UNIFORM || fire->mode == NCA_FIRE_THRESHOLD_UNIFORM) &&
      !fire->uniforms)
    return NCA_ERR_INVALID;
  if (fire->mode < 0 || fire->mode > 5) return NCA_ERR_INVALID;
  if (n_steps == 0) return NCA_OK;
  const bool split = st->precision == NCA_PREC_SPLIT;
  cudaStream_t s = as_stream(stream);
  const int C = m->channels, HD = m->hidden;
  if (fire->noise_mode < 0 || fire->noise_mode > 2) return NCA_ERR_INVALID;
  if (fire->noise_mode == NCA_NOISE_EXTERNAL && (!fire->noise || n_steps != 1)) return NCA_ERR_INVALID;
  const bool noise = fire->noise_mode != NCA_NOISE_NONE;
  const bool adaptive = fire->mode >= NCA_FIRE_ADAPTIVE_PHILOX;  // fire decisions on the confidence
  // Fire probabilities of the current state for the first step of each launch (the step kernel
  // keeps them up to date for the following steps).
  auto init_fire_p = [&]() -> int32_t {
    ReadoutArgs R;
    memset(&R, 0, sizeof(R));
    R.C = st->channels;
    R.hw = st->hw;
    R.n_inst = st->n_inst;
    R.c_out = m->c_out;
    R.out_off = m->out_offset;
    R.n_out = m->n_out;
    R.head_kind = m->head_kind;
    copy_head(R.head_w, R.head_b, m->head_w, m->head_b, m->n_out, m->c_out);
    const long long cells = st->n_tiles * kTileM;
    fire_p_kernel<<<(unsigned)((cells + 255) / 256), 256, 0, s>>>(
        st->master[st->cur], st->mirror[st->cur], st->channels, cells, (long long)st->n_inst * st->hw,
        st->hw, *b, R, fire->mode, fire->adapt_scale, fire->adapt_bias, fire->p_low, fire->tau,
        fire->p_fire, fire->given_confident, st->fire_p);
    return cuda_status(cudaGetLastError());
  };
  auto launch = [&](int32_t n, const NcaFireDesc* f) -> int32_t {
    if (adaptive) {
      const int32_t r = init_fire_p();
      if (r != NCA_OK) return r;
    }
    // the benchmark models (32, 128), (64, 256) and the reference's maze presets (16, 128),
    // (32, 256) (maze_ood, maze_hard: src/nca/model.py:656-700)
    if (C == 32 && HD == 128) return launch_shape_32_128(split, noise, adaptive, m, b, st, n, f, ctrl, timeout_ms, s);
    if (C == 64 && HD == 256) return launch_shape_64_256(split, noise, adaptive, m, b, st, n, f, ctrl, timeout_ms, s);
    if (C == 16 && HD == 128) return launch_shape_16_128(split, noise, adaptive, m, b, st, n, f, ctrl, timeout_ms, s);
    if (C == 32 && HD == 256) return launch_shape_32_256(split, noise, adaptive, m, b, st, n, f, ctrl, timeout_ms, s);
    return NCA_ERR_UNSUPPORTED;
  };
  if (st->clamped) return launch(n_steps, fire);
  // A state from outside the library: the first step runs alone and is followed by the clamp
  // of its output, as the reference clamps after every step; the remaining steps continue.
  int32_t r = launch(1, fire);
  if (r != NCA_OK) return r;
  const long long total = (long long)st->n_inst * st->hw;
  clamp_fix_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
      st->master[st->cur], st->mirror[st->cur], st->channels, total, st->hw, *b, m->c_in,
      m->in_offset);
  r = cuda_status(cudaGetLastError());
  if (r != NCA_OK) return r;
  st->clamped = 1;
  if (n_steps == 1) return NCA_OK;
  NcaFireDesc rest = *fire;
  rest.step0 += 1;
  if (rest.masks) rest.masks += total;
  if (rest.uniforms) rest.uniforms += total;
  return launch(n_steps - 1, &rest);
}

int32_t nca_b200_readout(const NcaModelDesc* m, const NcaBatchDesc* b, const NcaState* st,
                         uint8_t* pred, float* cell_conf, float* board_conf,
                         const uint8_t* targets, float* cell_acc, uint8_t* exact, void* stream) {
  if (!model_ok(m) || !batch_ok(b) || !st || !b->inputs) return NCA_ERR_INVALID;
  if (b->n_inst != st->n_inst || b->height * b->width != st->hw) return NCA_ERR_INVALID;
  ReadoutArgs R;
  memset(&R, 0, sizeof(R));
  R.C = st->channels;
  R.hw = st->hw;
  R.n_inst = st->n_inst;
  R.c_out = m->c_out;
  R.out_off = m->out_offset;
  R.n_out = m->n_out;
  R.head_kind = m->head_kind;
  copy_head(R.head_w, R.head_b, m->head_w, m->head_b, m->n_out, m->c_out);
  memcpy(R.out_tokens, m->out_tokens, sizeof(R.out_tokens));
  readout_kernel<<<st->n_inst, 128, 0, as_stream(stream)>>>(st->master[st->cur], st->mirror[st->cur], *b, R, pred,
                                                           cell_conf, board_conf, targets,
                                                           cell_acc, exact);
  return cuda_status(cudaGetLastError());
}

int32_t nca_b200_select(const float* board_conf, const uint8_t* alive, int32_t n_boards,
                        int32_t trials, int32_t k_limit, int32_t* best_idx, float* best_conf,
                        const uint8_t* pred, int32_t hw, uint8_t* best_pred, void* stream) {
  if (!board_conf || n_boards <= 0 || trials <= 0 || k_limit <= 0) return NCA_ERR_INVALID;
  if (k_limit > trials) k_limit = trials;
  const int threads = 256;
  const int blocks = (n_boards * 32 + threads - 1) / threads;
  select_kernel<<<blocks, threads, 0, as_stream(stream)>>>(board_conf, alive, n_boards, trials,
                                                           k_limit, best_idx, best_conf, pred, hw,
                                                           best_pred);
  return cuda_status(cudaGetLastError());
}

int32_t nca_b200_prune_refill(const uint8_t* pred, const float* board_conf, int32_t n_boards,
                              int32_t trials, int32_t hw, int32_t n_cap, int32_t* src,
                              uint8_t* kept, void* stream) {
  if (!pred || !board_conf || !src || n_boards <= 0 || trials <= 0 || hw <= 0 || n_cap < 1)
    return NCA_ERR_INVALID;
  if (trials > 1024) return NCA_ERR_UNSUPPORTED;
  const size_t sm = (size_t)trials * (8 + 4 + 4 + 4 + 4);
  const int threads = ((trials + 31) / 32) * 32;
  prune_refill_kernel<<<n_boards, threads, sm, as_stream(stream)>>>(pred, board_conf, trials, hw,
                                                                   n_cap, src, kept);
  return cuda_status(cudaGetLastError());
}

int32_t nca_b200_clone(NcaState* st, const int32_t* src, void* stream) {
  if (!st || !src) return NCA_ERR_INVALID;
  const bool hl = st->mirror[0] && hilo_layout(st->channels, true);
  const long long n = (long long)st->n_inst * st->hw * (st->channels / (hl ? 8 : 4));
  const int bs = 256;
  clone_kernel<<<(unsigned)((n + bs - 1) / bs), bs, 0, as_stream(stream)>>>(
      st->master[st->cur], st->mirror[st->cur], st->channels, st->hw, st->n_inst, src);
  return cuda_status(cudaGetLastError());
}

int32_t nca_b200_damage(const NcaModelDesc* m, const NcaBatchDesc* b, NcaState* st,
                        const uint8_t* masks, void* stream) {
  if (!model_ok(m) || !batch_ok(b) || !st || !masks) return NCA_ERR_INVALID;
  if (b->n_inst != st->n_inst || b->height * b->width != st->hw || m->channels != st->channels)
    return NCA_ERR_INVALID;
  const long long total = (long long)st->n_inst * st->hw;
  damage_kernel<<<(unsigned)((total + 255) / 256), 256, 0, as_stream(stream)>>>(
      st->master[st->cur], st->mirror[st->cur], st->channels, total, st->hw, *b, m->c_in,
      m->in_offset, masks);
  return cuda_status(cudaGetLastError());
}

int32_t nca_b200_niches(const uint8_t* pred, const float* board_conf, const int32_t* row_start,
                        int32_t n_boards, int32_t max_rows, int32_t hw, int32_t* niche,
                        int32_t* rank, int32_t* n_niches, void* stream) {
  if (!pred || !board_conf || !row_start || !niche || !rank || !n_niches || n_boards <= 0 ||
      max_rows <= 0 || hw <= 0)
    return NCA_ERR_INVALID;
  if (max_rows > 4096) return NCA_ERR_UNSUPPORTED;
  const size_t sm = (size_t)max_rows * (8 + 4 + 4 + 4);
  const int threads = max_rows < 1024 ? ((max_rows + 31) / 32) * 32 : 1024;
  niche_kernel<<<n_boards, threads, sm, as_stream(stream)>>>(pred, board_conf, row_start, hw,
                                                              max_rows, niche, rank, n_niches);
  return cuda_status(cudaGetLastError());
}

int32_t nca_b200_halving(const int32_t* niche, const int32_t* rank, const int32_t* n_niches,
                         const int32_t* row_start, const int32_t* order,
                         const int32_t* order_start, int32_t n_boards, int32_t max_rows,
                         int32_t n_cap, uint8_t* keep, void* stream) {
  if (!niche || !rank || !n_niches || !row_start || !order || !order_start || !keep ||
      n_boards <= 0 || max_rows <= 0 || n_cap < 1)
    return NCA_ERR_INVALID;
  if (max_rows > 4096) return NCA_ERR_UNSUPPORTED;
  const size_t sm = (size_t)max_rows * 8;
  const int threads = max_rows < 1024 ? ((max_rows + 31) / 32) * 32 : 1024;
  halving_kernel<<<n_boards, threads, sm, as_stream(stream)>>>(niche, rank, n_niches, row_start,
                                                                order, order_start, n_cap, max_rows, keep);
  return cuda_status(cudaGetLastError());
}

int32_t nca_b200_gather(const NcaState* src, NcaState* dst, const int32_t* sel, void* stream) {
  if (!src || !dst || !sel) return NCA_ERR_INVALID;
  if (src->channels != dst->channels || src->hw != dst->hw || src->precision != dst->precision ||
      dst->n_inst > src->n_inst)
    return NCA_ERR_INVALID;
  const bool hl = dst->mirror[0] && hilo_layout(dst->channels, true);
  const long long n = (long long)dst->n_inst * dst->hw * (dst->channels / (hl ? 8 : 4));
  if (n > 0) {
    const int bs = 256;
    gather_kernel<<<(unsigned)((n + bs - 1) / bs), bs, 0, as_stream(stream)>>>(
        src->master[src->cur], src->mirror[src->cur], dst->master[dst->cur], dst->mirror[dst->cur],
        dst->channels, dst->hw, dst->n_inst, sel);
  }
  dst->clamped = src->clamped;
  return cuda_status(cudaGetLastError());
}

int32_t nca_b200_resident_group(const NcaModelDesc* m, int32_t height, int32_t width) {
  if (!m || height < 1 || width < 1) return 0;
  const long long hw = (long long)height * width;
  if (m->channels == 32 && m->hidden == 128) return resident_capacity_32_128(hw);
  if (m->channels == 16 && m->hidden == 128) return resident_capacity_16_128(hw);
  if (m->channels == 32 && m->hidden == 256) return resident_capacity_32_256(hw);
  return 0;
}

int32_t nca_b200_ctrl_status(int32_t* ctrl, int32_t* detail, void* stream) {
  if (!ctrl) return NCA_ERR_INVALID;
  cudaStream_t s = as_stream(stream);
  int32_t h[4] = {0, 0, 0, 0};
  cudaError_t e = cudaMemcpyAsync(h, ctrl, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return NCA_ERR_CUDA;
  if (detail) *detail = h[1];
  if (h[0] != 0) {
    e = cudaMemsetAsync(ctrl, 0, sizeof(h), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return NCA_ERR_CUDA;
    return h[0];
  }
  return NCA_OK;
}

int32_t nca_b200_selftest_timeout(int32_t* ctrl, int32_t timeout_ms, void* stream) {
  if (!ctrl || timeout_ms <= 0) return NCA_ERR_INVALID;
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemsetAsync(ctrl, 0, 4 * sizeof(int32_t), s);
  if (e != cudaSuccess) return NCA_ERR_CUDA;
  selftest_wait_kernel<<<1, 64, 0, s>>>(ctrl, (unsigned long long)timeout_ms * 1000000ull);
  e = cudaGetLastError();
  if (e != cudaSuccess) return NCA_ERR_CUDA;
  return nca_b200_ctrl_status(ctrl, nullptr, stream);
}

}  // extern "C"

// ------------------------------------------------------------------------------------------
// Stepping without device allocation: the scratch of nca_b200_run_steps lives in this array.
namespace {

__device__ __align__(256) uint8_t g_static_scratch[NCA_B200_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
// Per device, the address of g_static_scratch, looked up on the first call with the device
// current.  Atomic: host threads that make a first call together each look it up and store the
// same value.  A cudaDeviceReset can move the module, so the kept address is valid only until a
// reset (documented in the header).
std::atomic<void*> g_static_scratch_addr[kMaxDevices];

// Device address of g_static_scratch on the current device (looked up once per device).
int32_t static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return NCA_ERR_DEVICE;
  void* p = g_static_scratch_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || p == nullptr)
      return NCA_ERR_CUDA;
    g_static_scratch_addr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return NCA_OK;
}

}  // namespace

extern "C" int32_t nca_b200_run_steps_static(const NcaModelDesc* m, const NcaBatchDesc* b,
                                             int32_t state_precision, const float* x_in,
                                             float* x_out, int32_t n_steps,
                                             const NcaFireDesc* fire, int32_t timeout_ms,
                                             void* stream) {
  if (!model_ok(m) || !batch_ok(b) || !fire || !x_in || !x_out || n_steps < 0) return NCA_ERR_INVALID;
  size_t need = 0;
  int32_t s = nca_b200_state_bytes(b->n_inst, b->height * b->width, m->channels, state_precision, &need);
  if (s != NCA_OK) return s;
  constexpr size_t kCtrlBytes = 256;  // control words, padded to keep the state 256-B aligned
  if (need + kCtrlBytes > (size_t)NCA_B200_STATIC_SCRATCH_BYTES) return NCA_ERR_SCRATCH;
  void* base = nullptr;
  s = static_scratch(&base);
  if (s != NCA_OK) return s;
  int32_t* ctrl = reinterpret_cast<int32_t*>(base);
  cudaStream_t st_ = as_stream(stream);
  if (cudaMemsetAsync(ctrl, 0, 4 * sizeof(int32_t), st_) != cudaSuccess) return NCA_ERR_CUDA;
  NcaState st;
  s = nca_b200_state_bind(&st, reinterpret_cast<uint8_t*>(base) + kCtrlBytes, need, b->n_inst,
                          b->height * b->width, m->channels, state_precision);
  if (s != NCA_OK) return s;
  s = nca_b200_state_load_nchw(&st, x_in, stream);
  if (s != NCA_OK) return s;
  s = nca_b200_run_steps(m, b, &st, n_steps, fire, ctrl, timeout_ms, stream);
  if (s != NCA_OK) return s;
  s = nca_b200_state_store_nchw(&st, x_out, stream);
  if (s != NCA_OK) return s;
  return nca_b200_ctrl_status(ctrl, nullptr, stream);
}
