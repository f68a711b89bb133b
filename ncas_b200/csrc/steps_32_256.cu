// steps_32_256.cu -- the step kernel instances of the (channels 32, hidden 256) model shape:
// bf16 / split precision x state noise x adaptive fire rules (x grid barrier / per-tile step
// counters inside launch_steps).  A translation unit of its own so that the shapes compile in
// parallel.
#include "launch.cuh"

namespace nca {

int32_t launch_shape_32_256(bool split, bool noise, bool adaptive, const NcaModelDesc* m,
                           const NcaBatchDesc* b, NcaState* st, int32_t n, const NcaFireDesc* f,
                           int32_t* ctrl, int32_t timeout_ms, cudaStream_t s) {
#define NCA_AD(SP, NZ)                                                                            \
  return adaptive ? launch_steps<StepCfg<32, 256, SP, NZ, false, true>>(m, b, st, n, f, ctrl, timeout_ms, s) \
                  : launch_steps<StepCfg<32, 256, SP, NZ>>(m, b, st, n, f, ctrl, timeout_ms, s);
  if (!split && !noise && !adaptive && f->resident && n > 1) {
    // the shared-memory-resident kernel, when a group of instances fits
    const int32_t r = launch_steps<StepCfg<32, 256, false, false, false, false, true>>(m, b, st, n, f, ctrl, timeout_ms, s);
    if (r != NCA_ERR_UNSUPPORTED) return r;
  }
  if (noise) {
    if (split) { NCA_AD(true, true) }
    NCA_AD(false, true)
  }
  if (split) { NCA_AD(true, false) }
  NCA_AD(false, false)
#undef NCA_AD
}

int32_t resident_capacity_32_256(long long hw) {
  return resident_capacity<StepCfg<32, 256, false, false, false, false, true>>(hw);
}

}  // namespace nca
