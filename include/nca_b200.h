/*
 * nca_b200.h -- C ABI of the B200 (sm_100a) Neural Cellular Automaton rollout library.
 *
 * The library replaces the test-time rollout hot path of JorisViaudQuantAI/NCAs (a Python /
 * PyTorch project).  Every entry point below names the reference function or method whose
 * work it performs; paths are relative to the reference repository root.
 *
 * Conventions
 *  - All pointers marked "device" point to CUDA device memory of the current device.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).  All work is
 *    enqueued on that stream; no call synchronises unless it says so.
 *  - Return values are NcaStatus codes.  Kernel-side failures (a bounded wait that ran out, a
 *    bounds check) are written to the caller's control words (`ctrl`, 4 x int32, device) and
 *    reported by nca_b200_ctrl_status().
 *  - No entry point allocates device memory: the caller provides every buffer, sized by the
 *    *_bytes() queries.
 *
 * State layout.  The reference keeps the state as fp32 NCHW (B, C, H, W).  Inside the library
 * a state lives in an NcaState workspace: cells are numbered g = inst * H * W + (i * W + j),
 * grouped into tiles of 128 cells, and stored as [tile][channel/4][128][4] fp32 ("master") plus
 * an optional bf16 copy [tile][channel/8][128][8] ("mirror") that feeds the perception stencil
 * in NCA_PREC_BF16 mode.  Both exist twice (ping-pong between steps).
 */
#ifndef NCA_B200_H
#define NCA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NCA_B200_ABI_VERSION 3
#define NCA_B200_MAX_OUT 16   /* maximum number of readout tokens (n_out) and readout channels */

typedef enum NcaStatus {
  NCA_OK = 0,
  NCA_ERR_INVALID = 1,      /* bad argument (null pointer, size mismatch) */
  NCA_ERR_UNSUPPORTED = 2,  /* a configuration the kernels do not implement */
  NCA_ERR_CUDA = 3,         /* a CUDA runtime call failed */
  NCA_ERR_TIMEOUT = 4,      /* a bounded wait inside a kernel ran out (see ctrl words) */
  NCA_ERR_DEVICE = 5,       /* no sm_100 device, or the kernel image does not load */
  NCA_ERR_KERNEL = 6,       /* a kernel reported an internal check failure (see ctrl words) */
  NCA_ERR_SCRATCH = 7       /* request larger than the static scratch of nca_b200_run_steps_static */
} NcaStatus;

typedef enum NcaPrecision {
  NCA_PREC_BF16 = 0,   /* bf16 tcgen05 GEMMs, bf16 stencil source (throughput mode) */
  NCA_PREC_SPLIT = 1   /* GEMM operands split into bf16 hi + lo parts, fp32 stencil (parity) */
} NcaPrecision;

typedef enum NcaFireMode {
  NCA_FIRE_MASK = 0,              /* external {0,1} masks [n_steps][n_inst][H*W] uint8 */
  NCA_FIRE_PHILOX = 1,            /* u < p_fire, u from in-kernel Philox4x32-10 */
  NCA_FIRE_ADAPTIVE_PHILOX = 2,   /* u < scale * (1 - conf) + bias, u from Philox */
  NCA_FIRE_ADAPTIVE_UNIFORM = 3,  /* same rule, u from external uniforms [n_steps][n_inst][H*W] */
  NCA_FIRE_THRESHOLD_PHILOX = 4,  /* the reference's threshold rule (src/nca/model.py:566-593):
                                     u < (conf > tau || given && given_confident ? p_low :
                                     p_fire), u from Philox */
  NCA_FIRE_THRESHOLD_UNIFORM = 5  /* same rule, u from external uniforms */
} NcaFireMode;

/* The cell rule: KernelPerception (4 heads of 3x3 taps, zero padding) + MLPUpdate + mlp head.
 * Mirrors nca.model.NCAConfig / NCA (src/nca/model.py:48-137, 161-178, 277-287, 344-345). */
typedef struct NcaModelDesc {
  int32_t channels;     /* C: 16, 32 or 64 */
  int32_t perception;   /* P = 4 * C (heads = 4) */
  int32_t hidden;       /* Hd: multiple of 32, <= 256 */
  int32_t c_in, in_offset;    /* clamped input slice [in_offset, in_offset + c_in) */
  int32_t c_out, out_offset;  /* readout slice [out_offset, out_offset + c_out) */
  int32_t n_out;              /* number of readout tokens */
  int32_t fixed_taps;         /* 1: taps are identity, Sobel-x, Sobel-y, Laplacian (fast path) */
  float taps[4][9];           /* perceive.weight (heads, 1, 3, 3), row-major taps */
  float head_w[NCA_B200_MAX_OUT][NCA_B200_MAX_OUT]; /* head.weight[o][c] (n_out x c_out) */
  float head_b[NCA_B200_MAX_OUT];
  int32_t out_tokens[NCA_B200_MAX_OUT];             /* nca.model.NCAConfig.output_tokens */
  const void* weights;  /* device: image written by nca_b200_pack_weights + uploaded */
  const float* b1;      /* device [hidden]   update.fc1.bias */
  const float* b2;      /* device [channels] update.fc2.bias */
  int32_t head_kind;    /* NCA_HEAD_LINEAR: scores head_w x + head_b, softmax confidence
                           (head "mlp"); NCA_HEAD_L2: head_w rows are the output-token embeddings
                           (out_embed), score 1 / (1 + |x - e|), confidence the best score
                           (src/nca/model.py:596-633) */
  float pad[64];        /* state of the cells outside the board by channel: the wall token's
                           embedding for wall padding (pad_vec, src/nca/model.py:140-152, 320-325),
                           zeros for zero padding */
  const void* weights_lo;  /* optional device image (same layout as `weights`) of the residual
                              w - bf16(w): NCA_PREC_SPLIT then computes the GEMMs with fp32-accurate
                              weights (trained fp32 checkpoints); NULL when the weights are bf16 */
} NcaModelDesc;

typedef enum NcaHeadKind { NCA_HEAD_LINEAR = 0, NCA_HEAD_L2 = 1 } NcaHeadKind;

/* A batch of instances (board x trial rows of the reference's flattened batch,
 * src/nca/rollout.py:144-150).  Instance `inst` uses clamp row inst_row[inst], or inst / trials
 * when inst_row is NULL. */
typedef struct NcaBatchDesc {
  int32_t n_inst, height, width;
  int32_t trials;           /* K */
  int64_t inst_offset;      /* global index of instance 0 (Philox counters; shards agree) */
  const uint8_t* given;     /* device [rows][H*W] 1 = clamped cell (given4) */
  const float* clamp;       /* device [rows][H*W][c_in] clamp values (embedding of the input) */
  const uint8_t* inputs;    /* device [rows][H*W] input tokens (readout fills given cells) */
  const int32_t* inst_row;  /* optional device [n_inst]: board row of each instance (default
                               instance / trials) */
  const int32_t* inst_id;   /* optional device [n_inst]: trial identity of each instance for the
                               Philox counters (default the instance index), so a trial keeps its
                               random stream when a compacted batch renumbers it */
} NcaBatchDesc;

typedef struct NcaState {
  int32_t n_inst, hw, channels, precision;
  int64_t n_tiles;          /* ceil(n_inst * hw / 128) */
  float* master[2];         /* device, tiled fp32 */
  uint16_t* mirror[2];      /* device, tiled bf16 (NULL in NCA_PREC_SPLIT) */
  int32_t cur;              /* index of the buffers holding the current state */
  int32_t clamped;          /* 1 when the given cells of the current state hold their clamp
                               values (set by nca_b200_state_init and by every step; cleared by
                               nca_b200_state_bind and nca_b200_state_load_nchw) */
  uint32_t* tile_steps;     /* device [n_tiles]: per-tile step counters of a launch (the step
                               kernel's dependencies between neighbouring tiles) */
  float* fire_p;            /* device [n_tiles * 128]: per cell, the fire probability of the next
                               step under the confidence rules (fire modes 2..5), written before
                               and during a launch */
} NcaState;

typedef enum NcaNoiseMode {
  NCA_NOISE_NONE = 0,
  NCA_NOISE_PHILOX = 1,     /* in-kernel: Philox draws for instance, cell and Gaussian values */
  NCA_NOISE_EXTERNAL = 2    /* caller's noise tensor (the reference's torch stream) */
} NcaNoiseMode;

typedef struct NcaFireDesc {
  int32_t mode;             /* NcaFireMode */
  float p_fire;             /* RolloutConfig.fire_rate */
  float adapt_scale, adapt_bias;  /* p = scale * (1 - conf_cell) + bias */
  float p_low, tau;         /* threshold rule: RolloutConfig.p_low, RolloutConfig.tau */
  int32_t given_confident;  /* threshold rule: given cells count as confident */
  uint64_t seed;            /* Philox key */
  int64_t step0;            /* absolute index of the first step of this call */
  const uint8_t* masks;     /* device [n_steps][n_inst][H*W] (NCA_FIRE_MASK) */
  const float* uniforms;    /* device [n_steps][n_inst][H*W] (NCA_FIRE_ADAPTIVE_UNIFORM) */
  uint32_t* updates;        /* optional device [n_inst]: fired cells are added here */
  /* Test-time state noise (src/nca/perturb.py:23-40, added after the update and before the
   * clamp, src/nca/model.py:544-546), on steps with absolute index < noise_until: */
  int32_t noise_mode;       /* NcaNoiseMode */
  float noise_p_t;          /* probability that an instance is perturbed at a step */
  float noise_p_s;          /* probability that a cell of a perturbed instance is */
  float noise_sigma;        /* standard deviation of the Gaussian values */
  int64_t noise_until;
  const float* noise;       /* NCA_NOISE_EXTERNAL: device [n_inst][C][H*W] noise of the single
                               step of the call (n_steps must be 1) */
  int32_t resident;         /* 1: run the steps with each instance's state resident in shared
                               memory when whole instances fit (bf16 precision, fewer than 64
                               channels, no noise or confidence rules, n_steps > 1): the state is
                               kept as bf16 hi + lo parts between the steps of the call and read
                               from / written to HBM once; 0 (or when it does not apply): the
                               streaming kernel, one HBM round trip per step */
} NcaFireDesc;

/* ---- library / device --------------------------------------------------------------------- */
int32_t nca_b200_abi_version(void);
const char* nca_b200_status_string(int32_t status);
/* Checks that `device` is an sm_100 part and that the kernels load on it. */
int32_t nca_b200_device_info(int32_t device, int32_t* sm_count, int32_t* cc_major,
                             int32_t* cc_minor);

/* ---- weights ------------------------------------------------------------------------------ */
/* Host-side: bytes of the packed bf16 weight image (fc1 then fc2, 128B-swizzled K-major). */
int32_t nca_b200_weights_bytes(int32_t channels, int32_t perception, int32_t hidden,
                               size_t* bytes);
/* Host-side packing of update.fc1.weight (hidden x perception) and update.fc2.weight
 * (channels x hidden), fp32 row-major, into the image.  Replaces the fp32->bf16 weight cast the
 * reference's Triton MLP does per call (src/nca/engine/triton_mlp.py:138-156). */
int32_t nca_b200_pack_weights(const float* w1, const float* w2, int32_t channels,
                              int32_t perception, int32_t hidden, void* image_host);

/* ---- state -------------------------------------------------------------------------------- */
int32_t nca_b200_state_bytes(int32_t n_inst, int32_t hw, int32_t channels, int32_t precision,
                             size_t* bytes);
/* Carves an NcaState out of a caller buffer of nca_b200_state_bytes() bytes (256-B aligned). */
int32_t nca_b200_state_bind(NcaState* st, void* buffer, size_t bytes, int32_t n_inst,
                            int32_t hw, int32_t channels, int32_t precision);
/* Zero state + clamp of the given cells: nca.model.NCA.init_state with sigma_init = 0
 * (src/nca/model.py:384-412, apply_clamp 430-438). */
int32_t nca_b200_state_init(NcaState* st, const NcaModelDesc* m, const NcaBatchDesc* b,
                            void* stream);
/* fp32 NCHW (n_inst, C, H, W) <-> NcaState.  The reference's state format
 * (src/nca/model.py:29-30). */
int32_t nca_b200_state_load_nchw(NcaState* st, const float* x_nchw, void* stream);
int32_t nca_b200_state_store_nchw(const NcaState* st, float* x_nchw, void* stream);

/* ---- the rollout step --------------------------------------------------------------------- */
/* n_steps NCA steps on every instance: perception stencil, MLP on tcgen05, fire mask, residual
 * update, clamp.  Replaces nca.model.NCA.step (src/nca/model.py:503-525, residual_update
 * 527-559, sample_fire_mask 567-593) looped by nca.rollout.rollout (src/nca/rollout.py:203-247)
 * and nca.engine.inference.UniformRolloutBlocks.__call__ (src/nca/engine/inference.py:98-104).
 * n_steps > 1 runs as one persistent cooperative launch with a bounded grid barrier per step.
 * `ctrl` is 4 x int32 device control words (error code, detail, barrier, abort). */
int32_t nca_b200_run_steps(const NcaModelDesc* m, const NcaBatchDesc* b, NcaState* st,
                           int32_t n_steps, const NcaFireDesc* fire, int32_t* ctrl,
                           int32_t timeout_ms, void* stream);
/* The shared-memory-resident form of the step (NcaFireDesc.resident): the number of whole
 * instances of a height x width board that one CTA keeps in shared memory for all steps of a
 * launch, 0 when the model's shape has no resident kernel (64 channels) or not even one instance
 * fits.  A launch with resident = 1 runs the resident kernel exactly when this is at least 1, the
 * state precision is bf16, the fire rule is not a confidence rule, there is no state noise and
 * n_steps > 1; the state is then read once and written once per launch.  An addition of this
 * library (the reference steps every batch through global memory). */
int32_t nca_b200_resident_group(const NcaModelDesc* m, int32_t height, int32_t width);

/* ---- readout, selection, pruning ---------------------------------------------------------- */
/* Per cell: argmax token of the mlp head (given cells show their input token) and max-softmax
 * confidence; per instance: mean confidence over all H*W cells and, with `targets`, the
 * fraction of mutable cells correct and the exact flag.  Replaces NCA.decode / confidence /
 * board_confidence (src/nca/model.py:596-633), decode_boards (src/nca/rollout.py:74-82) and the
 * rollout's score() (src/nca/rollout.py:181-184).  Any output pointer may be NULL. */
int32_t nca_b200_readout(const NcaModelDesc* m, const NcaBatchDesc* b, const NcaState* st,
                         uint8_t* pred, float* cell_conf, float* board_conf,
                         const uint8_t* targets, float* cell_acc, uint8_t* exact,
                         void* stream);
/* conf@K selection: per board the first index of the largest confidence among alive trials
 * k < k_limit (np.argmax semantics), its confidence and (optionally) its decoded grid.
 * Replaces the selection inside nca.rollout.conf_at_k (src/nca/rollout.py:317-334). */
int32_t nca_b200_select(const float* board_conf, const uint8_t* alive, int32_t n_boards,
                        int32_t trials, int32_t k_limit, int32_t* best_idx, float* best_conf,
                        const uint8_t* pred, int32_t hw, uint8_t* best_pred, void* stream);
/* Niche-capped pruning with refill: trials whose decoded grids are byte-identical form a niche
 * (grouping of src/nca/pruning.py:39-41); each niche keeps its n_cap most confident members
 * (stable sort, src/nca/pruning.py:43-46); every dropped slot is refilled with a clone of a
 * kept trial, kept trials taken in decreasing confidence, cycling.  Writes src[inst] (the
 * instance whose state slot `inst` continues from) and kept[inst]. */
int32_t nca_b200_prune_refill(const uint8_t* pred, const float* board_conf, int32_t n_boards,
                              int32_t trials, int32_t hw, int32_t n_cap, int32_t* src,
                              uint8_t* kept, void* stream);
/* Copies the state of instance src[i] into instance i wherever src[i] != i (the batch gather
 * x[sel] of src/nca/rollout.py:270-274, without compaction).  In place: every source must map to
 * itself (src[src[i]] == src[i]), as the maps written by nca_b200_prune_refill do. */
int32_t nca_b200_clone(NcaState* st, const int32_t* src, void* stream);

/* Damage event (src/nca/rollout.py:206-212, src/nca/perturb.py:43-83): every channel of the
 * cells with masks[row][cell] != 0 is set to zero in every instance of that board row, then the
 * clamp of the given cells is applied again (src/nca/model.py:430-438).  masks: device
 * [rows][H*W] uint8 (the reference's circular_masks, one per board). */
int32_t nca_b200_damage(const NcaModelDesc* m, const NcaBatchDesc* b, NcaState* st,
                        const uint8_t* masks, void* stream);

/* Niche-Capped Diversity Pruning, halving variant (src/nca/pruning.py:22-65), in two calls
 * around the host's random draws.  The alive trials of board n are the rows
 * [row_start[n], row_start[n + 1]) of a compacted batch, in increasing trial order.
 * nca_b200_niches groups them by identical decoded grid (pruning.py:39-41): niche[r] is the index
 * of the niche of row r in order of first appearance, rank[r] its position in the niche by
 * decreasing confidence (stable, pruning.py:43-46), n_niches[n] the board's niche count.
 * The host then draws the niche order of every board with more than one alive trial
 * (rng.permutation(n_niches[n]), pruning.py:48), concatenated in `order` from order_start[n].
 * nca_b200_halving keeps floor(alive / 2) rows per board, taken round-robin over the niches in
 * that order, most confident first, at most n_cap per niche (pruning.py:49-61): keep[r]. */
int32_t nca_b200_niches(const uint8_t* pred, const float* board_conf, const int32_t* row_start,
                        int32_t n_boards, int32_t max_rows, int32_t hw, int32_t* niche,
                        int32_t* rank, int32_t* n_niches, void* stream);
int32_t nca_b200_halving(const int32_t* niche, const int32_t* rank, const int32_t* n_niches,
                         const int32_t* row_start, const int32_t* order,
                         const int32_t* order_start, int32_t n_boards, int32_t max_rows,
                         int32_t n_cap, uint8_t* keep, void* stream);
/* Compaction of a batch (x[sel] of src/nca/rollout.py:262-274): instance i of dst receives the
 * current state of instance sel[i] of src, for i < dst->n_inst.  Both states have the same
 * channels, cells and precision; dst is a separate workspace. */
int32_t nca_b200_gather(const NcaState* src, NcaState* dst, const int32_t* sel, void* stream);

/* ---- control words ------------------------------------------------------------------------ */
/* Synchronises `stream`, reads the control words and returns NCA_OK or the first kernel-side
 * error; detail (may be NULL) receives the failing site.  Clears the words on return. */
int32_t nca_b200_ctrl_status(int32_t* ctrl, int32_t* detail, void* stream);
/* Self-test of the bounded waits: launches a kernel that waits for a flag nothing sets, with
 * the given timeout; returns NCA_ERR_TIMEOUT (the expected result) when the wait gave up. */
int32_t nca_b200_selftest_timeout(int32_t* ctrl, int32_t timeout_ms, void* stream);

/* ---- stepping without any device allocation ---------------------------------------------- */
/* Size of the library's file-scope device array used by nca_b200_run_steps_static: 16 MiB.  Every
 * GPU that loads the library holds it until the process exits. */
#define NCA_B200_STATIC_SCRATCH_BYTES (16u << 20)

/* For callers that cannot allocate device memory: a host framework whose allocator owns all
 * device memory and hands out only the caller's tensors, or an embedded runtime with a fixed
 * device-memory budget fixed at start-up.  It runs the same n_steps as nca_b200_run_steps, but
 * the kernel's scratch (the ping-pong state workspace and the four control words) lives in a
 * static 16 MiB device array inside the library instead of buffers the caller allocates; the
 * caller passes only inputs and outputs: the fp32 NCHW state before (x_in) and after (x_out) the
 * steps, both n_inst x channels x H x W.
 *  - Limit: nca_b200_state_bytes(n_inst, H*W, channels, state_precision) + 256 bytes must fit in
 *    NCA_B200_STATIC_SCRATCH_BYTES, else NCA_ERR_SCRATCH (e.g. 32,000 Sudoku cells at C = 64 or one
 *    201 x 201 maze at C = 32 in bf16 mode).
 *  - It calls no allocator.  Its first call on a device looks up the device address of the array
 *    (cudaGetSymbolAddress with that device current) and keeps it for the process; make that
 *    first call before any stream capture on the device.  Two host threads making a first call
 *    on one device at the same time both look the address up and store the same value.  After a
 *    cudaDeviceReset the kept address may be stale: do not use this entry point after a reset.
 *  - All calls share the one array, which keeps the last call's contents; the call clears the
 *    control words and rewrites the state workspace before use.  Calls that overlap on the GPU
 *    (other streams, other host threads) race on the array: serialise them.
 *  - It waits for its own work: the stream is synchronised before it returns, so that a kernel
 *    timeout comes back as NCA_ERR_TIMEOUT.  It returns the status code only: the failing site
 *    that nca_b200_ctrl_status reports through `detail` is not available here.
 * There is no counterpart in the reference: it is an addition of this library. */
int32_t nca_b200_run_steps_static(const NcaModelDesc* m, const NcaBatchDesc* b,
                                  int32_t state_precision, const float* x_in, float* x_out,
                                  int32_t n_steps, const NcaFireDesc* fire, int32_t timeout_ms,
                                  void* stream);

#ifdef __cplusplus
}
#endif
#endif /* NCA_B200_H */
