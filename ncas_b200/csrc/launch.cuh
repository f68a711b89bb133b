// launch.cuh -- host-side launch of the persistent step kernel for one StepCfg: builds the
// kernel arguments from the C-ABI descriptors, sizes the window stages to the shared memory,
// chooses grid barrier or per-tile step counters, and launches (cooperatively when the launch
// runs more than one step).  Included by the per-shape translation units (steps_*.cu), which
// instantiate it for the kernel shapes the library exports.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/nca_b200.h"
#include "step_kernel.cuh"

namespace nca {

constexpr int kMaxSmem = 232448;  // opt-in dynamic shared memory per CTA on sm_100

// Resident kernel: the most whole instances of `hw` cells one CTA keeps in shared memory (the
// two buffers of hi parts, the lo parts and the weights), 0 when not even one fits.
template <class Cfg>
inline int32_t resident_capacity(long long hw) {
  static_assert(Cfg::RESIDENT, "resident kernel shapes only");
  if (hw < 1 || hw > kMaxSmem) return 0;
  auto smem_for = [&](long long inst) { return SmemLayout<Cfg>(2, (int)(inst * hw), false).total + 1024LL; };
  int32_t g = 0;
  while (smem_for(g + 1) <= kMaxSmem) ++g;
  return g;
}

template <class Cfg>
inline int32_t launch_steps(const NcaModelDesc* m, const NcaBatchDesc* b, NcaState* st, int32_t n_steps,
                     const NcaFireDesc* fire, int32_t* ctrl, int32_t timeout_ms,
                     cudaStream_t stream) {
  StepArgs A;
  memset(&A, 0, sizeof(A));
  A.n_inst = b->n_inst;
  A.H = b->height;
  A.W = b->width;
  A.HW = b->height * b->width;
  A.K = b->trials;
  A.div_hw = make_fastdiv((unsigned)A.HW);
  A.div_w = make_fastdiv((unsigned)A.W);
  A.div_k = make_fastdiv((unsigned)A.K);
  A.total = (long long)b->n_inst * A.HW;
  if (A.total + 2 * kTileM + 2LL * A.W >= (1LL << 31)) return NCA_ERR_UNSUPPORTED;  // 32-bit cell ids
  A.n_tiles = st->n_tiles;
  A.inst_offset = b->inst_offset;
  A.n_steps = n_steps;
  A.step0 = fire->step0;
  A.win_cells = kTileM + 2 * b->width + 2;
  A.c_in = m->c_in;
  A.in_off = m->in_offset;
  A.c_out = m->c_out;
  A.out_off = m->out_offset;
  A.n_out = m->n_out;
  A.fixed_taps = m->fixed_taps;
  memcpy(A.taps, m->taps, sizeof(A.taps));
  copy_head(A.head_w, A.head_b, m->head_w, m->head_b, m->n_out, m->c_out);
  A.wimg = reinterpret_cast<const uint8_t*>(m->weights);
  A.wimg_lo = (st->precision == NCA_PREC_SPLIT) ? reinterpret_cast<const uint8_t*>(m->weights_lo) : nullptr;
  A.head_kind = m->head_kind;
  memcpy(A.pad, m->pad, sizeof(A.pad));
  A.b1 = m->b1;
  A.b2 = m->b2;
  A.given = b->given;
  A.clamp = b->clamp;
  A.inst_row = b->inst_row;
  A.inst_id = b->inst_id;
  A.master[0] = st->master[0];
  A.master[1] = st->master[1];
  A.mirror[0] = st->mirror[0];
  A.mirror[1] = st->mirror[1];
  A.cur = st->cur;
  A.fire_mode = fire->mode;
  A.p_fire = fire->p_fire;
  A.ad_scale = fire->adapt_scale;
  A.ad_bias = fire->adapt_bias;
  A.p_low = fire->p_low;
  A.tau = fire->tau;
  A.given_confident = fire->given_confident;
  A.seed = fire->seed;
  A.masks = fire->masks;
  A.uniforms = fire->uniforms;
  A.updates = fire->updates;
  A.noise_mode = fire->noise_mode;
  A.noise_p_t = fire->noise_p_t;
  A.noise_p_s = fire->noise_p_s;
  A.noise_sigma = fire->noise_sigma;
  A.noise_until = fire->noise_until;
  A.noise = fire->noise;
  A.ctrl = ctrl;
  A.timeout_ns = (unsigned long long)(timeout_ms > 0 ? timeout_ms : 10000) * 1000000ull;

  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return NCA_ERR_CUDA;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return NCA_ERR_CUDA;

  int stages, smem;
  long long grid_ll;
  if constexpr (Cfg::RESIDENT) {
    // Groups of whole instances: as many as fit the shared memory (the two hi buffers and the lo
    // parts), but no more than spread the batch over every SM.
    if (n_steps < 2 || A.total + 2LL * kTileM >= (1LL << 31)) return NCA_ERR_UNSUPPORTED;
    long long g_cap = resident_capacity<Cfg>(A.HW);
    if (g_cap > A.n_inst) g_cap = A.n_inst;
    if (g_cap < 1) return NCA_ERR_UNSUPPORTED;
    const long long spread = (A.n_inst + sms - 1) / sms;
    const long long g = g_cap < spread ? g_cap : spread;
    A.res_inst = (int)g;
    A.res_cells = g * A.HW;
    A.n_groups = (A.n_inst + g - 1) / g;
    stages = 2;
    A.win_cells = (int)A.res_cells;  // the padding cell follows the group's cells
    smem = SmemLayout<Cfg>(2, (int)A.res_cells, false).total + 1024;
    grid_ll = A.n_groups < sms ? A.n_groups : sms;
  } else {
    // Window stages: in the hi/lo layout a window lives from the stencil to the epilogue (which
    // reads the hi part of the old state from it), so more stages keep the stencil ahead.
    stages = Cfg::HILO ? kMaxStages : 2;
    smem = SmemLayout<Cfg>(stages, A.win_cells, A.wimg_lo != nullptr).total + 1024;
    while (smem > kMaxSmem && stages > 1) {
      --stages;
      smem = SmemLayout<Cfg>(stages, A.win_cells, A.wimg_lo != nullptr).total + 1024;
    }
    if (smem > kMaxSmem) return NCA_ERR_UNSUPPORTED;
    grid_ll = A.n_tiles < sms ? A.n_tiles : sms;
  }
  A.stages = stages;
  const int grid = (int)(grid_ll > 0 ? grid_ll : 1);
  // Steps are ordered by per-tile step counters when every CTA has few tiles (a grid barrier
  // would idle the whole GPU at each step boundary), else by the grid barrier on ctrl[2], whose
  // cost is then small against the step (the per-tile form costs the epilogue registers and the
  // MMA warp a publisher lane).
  const bool tiledep = !Cfg::RESIDENT && n_steps > 1 && A.n_tiles <= (long long)kTileDepPerCta * grid;
  using CfgTD = StepCfg<Cfg::C, Cfg::HD, Cfg::SPLIT, Cfg::NOISE, !Cfg::RESIDENT, Cfg::ADAPTIVE, Cfg::RESIDENT>;
  auto kern = tiledep ? nca_step_kernel<CfgTD> : nca_step_kernel<Cfg>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return NCA_ERR_CUDA;

  A.tile_steps = tiledep ? st->tile_steps : nullptr;
  A.fire_p = st->fire_p;
  if (tiledep) {
    e = cudaMemsetAsync(st->tile_steps, 0, (size_t)st->n_tiles * sizeof(uint32_t), stream);
    if (e != cudaSuccess) return NCA_ERR_CUDA;
  }
  e = cudaMemsetAsync(ctrl + 2, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return NCA_ERR_CUDA;
  if (n_steps > 1 && !Cfg::RESIDENT) {  // the resident kernel's CTAs never wait for each other
    void* args[] = {&A};
    e = cudaLaunchCooperativeKernel((const void*)kern, dim3(grid), dim3(Cfg::THREADS), args,
                                    (size_t)smem, stream);
  } else {
    kern<<<grid, Cfg::THREADS, smem, stream>>>(A);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return NCA_ERR_CUDA;
  st->cur = (st->cur + n_steps) & 1;
  return NCA_OK;
}


// One (channels, hidden) shape: the eight instantiations of its fire / noise / precision modes.
// Defined in steps_<C>_<HD>.cu.
#define NCA_DECLARE_SHAPE(CC, HH)                                                                 \
  int32_t launch_shape_##CC##_##HH(bool split, bool noise, bool adaptive, const NcaModelDesc* m, \
                                   const NcaBatchDesc* b, NcaState* st, int32_t n,               \
                                   const NcaFireDesc* f, int32_t* ctrl, int32_t timeout_ms,      \
                                   cudaStream_t s);
NCA_DECLARE_SHAPE(32, 128)
NCA_DECLARE_SHAPE(64, 256)
NCA_DECLARE_SHAPE(16, 128)
NCA_DECLARE_SHAPE(32, 256)
#undef NCA_DECLARE_SHAPE

// resident_capacity of the shapes with a resident kernel (channels below 64)
int32_t resident_capacity_32_128(long long hw);
int32_t resident_capacity_16_128(long long hw);
int32_t resident_capacity_32_256(long long hw);

// The attributes of one step-kernel instance (checks that the kernel image loads on a device).
cudaError_t step_kernel_attributes(cudaFuncAttributes* fa);

}  // namespace nca
