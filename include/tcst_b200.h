/*
 * tcst_b200.h -- C ABI of the B200 (sm_100a) radius cell-mass Linear backend.
 *
 * The library computes the training hot path of a torchcst CSTLinear layer whose
 * kernel is product(cell_mass(ChebyshevSpec(M)), cell_mass(...)) on two 1-D
 * flat-torus regular grids with rational-radius or Polar-radius coordinates:
 *
 *     W[o,i] = sum_a amp_a m_out,a(o) m_in,a(i),   Y = X W^T,
 *
 * its backward (dX and atom-parameter gradients) and the fused CSTAdamW step.
 *
 * Conventions
 *   - Every pointer argument named *_dev is CUDA device memory of the current
 *     device; nothing here allocates device memory. Sizes are element counts.
 *   - `stream` is a cudaStream_t passed as void*; NULL means the legacy stream.
 *     It belongs to the current device. The weight assembly and pullback entry
 *     points fork independent kernels onto internal side streams of that device
 *     and join them back to `stream` before returning (event records and waits
 *     only: the work completes in `stream` order and can be graph-captured).
 *   - The atom table is 16-byte aligned (checked).
 *   - Every function returns TCST_OK (0) or a nonzero TCST_ERR_* code; the text
 *     of the most recent failure on the calling host thread is returned by
 *     tcst_last_error().
 *   - Device-side validation never traps: kernels OR bits into a caller-owned
 *     device status word (TCST_STATUS_*), which the caller reads when it wants.
 *   - Matrices are row-major with an explicit leading dimension `ld` (elements).
 */
#ifndef TCST_B200_H
#define TCST_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TCST_OK 0
#define TCST_ERR_ARGUMENT 1    /* invalid sizes, pointers or declarations */
#define TCST_ERR_CUDA 2        /* a CUDA runtime/driver call failed */
#define TCST_ERR_UNSUPPORTED 3 /* a valid request outside this build's limits */

/* Bits of the device status word. */
#define TCST_STATUS_NONFINITE 1u     /* non-finite atom coordinate */
#define TCST_STATUS_BOUNDS 2u        /* rational q outside [0,1] or |a| > amplitude_max */
#define TCST_STATUS_RADIUS 4u        /* radius outside (0, chart period / 2] */
#define TCST_STATUS_TIMEOUT 8u       /* a bounded device wait gave up */
#define TCST_STATUS_FOOTPRINT 16u    /* footprint longer than this build supports */
#define TCST_STATUS_SEQUENCE 32u     /* a scalar ring slot did not hold the expected step */

#define TCST_RATIONAL 0
#define TCST_POLAR 1

/* One fixed 1-D flat-torus regular grid and its cell-mass hierarchy:
 * RadiusCellMassGrid (torchcst kernels/radius_cell_mass.py:16-26) plus the
 * RadiusIntegratedProfileBinding fields (kernels/spec.py:133-157) and
 * ChebyshevSpec.modes. The ratio site_count / base_tile_sites must be a power of
 * merge_factor. */
typedef struct tcst_axis {
    int32_t site_count;
    int32_t base_tile_sites;
    int32_t merge_factor;
    int32_t modes; /* Chebyshev modes M, 1..16 */
    double spacing;
    double origin;
} tcst_axis;

/* Atom coordinate law. kind = TCST_RATIONAL: rows [a, q, mu_out, mu_in]
 * (RationalRadiusSpec, kernels/parameterizations/rational_radius.py:9-32).
 * kind = TCST_POLAR: rows [s, t, mu_out, mu_in] with the rational radius
 * envelope (PolarAmpRadiusSpec, kernels/parameterizations/activity_width.py:68).
 * Values are the float32 KernelState scalars widened to double. Bounds arrays
 * are (minimum, birth, maximum, upper_floor). */
typedef struct tcst_coordinates {
    int32_t kind;
    int32_t reserved;
    double amplitude_max;
    double radius_min, radius_birth, radius_max;      /* rational */
    double w_c, kappa, lower_kappa, upper_decay_power; /* Polar */
    double out_bounds[4];
    double in_bounds[4];
} tcst_coordinates;

/* One CSTAdamW step (optim/adamw.py:230-294 with torch's single-tensor AdamW
 * numerics, optim/_field_lrs.py:128-134, and the coordinate law). Float fields
 * are the values torch casts its Python scalars to. */
typedef struct tcst_adamw {
    float lerp_weight;     /* 1 - beta1 */
    float beta2;           /* beta2 */
    float one_minus_beta2; /* 1 - beta2 */
    float neg_step_size;   /* -lr / (1 - beta1^step) */
    float bias2_sqrt;      /* sqrt(1 - beta2^step) */
    float eps;
    float decay_factor;    /* 1 - lr * weight_decay (used when has_decay) */
    int32_t has_decay;
    float field_ratio[4];  /* per column: field_lr / lr */
    int32_t field_mask;    /* bit c set: column c has a field ratio */
    /* coordinate law */
    float amplitude_cap;   /* rational: float32 amplitude_max, nudged inward */
    float polar_amplitude_max, polar_w_c;
    float polar_activity_gain, polar_dormant_q_scale; /* 3 * rate * lr */
    float polar_decay;     /* exp(-4 * radial_regularization * lr) in float32 */
    float polar_energy_step; /* lr for activity_mode time_energy, else 0 */
    float period_out, period_in;
    /* Polar decoupled amplitude decay after the activity law
     * (_backends/torch/algorithms/polar_update/executor.py:18-41): float32 of
     * lr * amplitude_weight_decay; 0 leaves the step unchanged. */
    float amplitude_decay;
} tcst_adamw;

const char *tcst_version(void);
const char *tcst_last_error(void);

/* Bytes of the atom table written by tcst_decode_route: per-atom records,
 * footprint spans, the site values of narrow footprints, the atoms sorted into
 * bins (footprint class x first-site tile, or owner pair for wide atoms of a
 * shared tile hierarchy; id order inside each bin) that the weight assembly and
 * the pullback walk, and the owner-pair region (per-pair 17 x 17 coefficient
 * matrices, node flags and the expansion buffers of the Fourier owner-pair
 * path, which the assembly and the pullback of the same table fill). */
int64_t tcst_atom_table_bytes(int64_t atoms, const tcst_axis *out_axis,
                              const tcst_axis *in_axis);

/* Decode coordinates, route every atom on both axes and evaluate its
 * Chebyshev-square Fourier profile. Replaces the decode/routing/profile part of
 * radius_cell_mass.factors (_backends/torch/kernels/radius_cell_mass.py:225-247,
 * :66-123; _backends/torch/profiles/radius_fourier.py:14-58;
 * _backends/torch/parameterizations/rational_radius.py:6-38) and the reference
 * CUDA classify_kernel (radius_cell_mass/pipeline.cu:43-81).
 * owner_keys_dev (nullable): no * input_node_count + ni per atom, as pipeline.cu:75-80.
 * routing_dev (nullable): [atoms][6] = out level, out K, out first tile, in level,
 * in K, in first tile. */
int tcst_decode_route(const float *p_dev, int64_t atoms, const tcst_axis *out_axis,
                      const tcst_axis *in_axis, const tcst_coordinates *coords,
                      void *atom_table_dev, int64_t *owner_keys_dev,
                      int32_t *routing_dev, uint32_t *status_dev, void *stream);

/* Assemble the dense weight W = sum_a amp_a m_out,a (x) m_in,a (images folded
 * modulo N) from the atom table. Replaces the W side of factors/weight
 * (radius_cell_mass.py:225-263). Each 32 x 32 tile of W gathers, in a fixed
 * order, the bins whose atoms can reach it; atoms of owner pairs with two or
 * more atoms come in through the pair's 17 x 17 Fourier coefficients instead
 * (the reference's wide-atom factorisation). W is bitwise reproducible.
 * scratch_dev is 16-byte aligned and tcst_weight_scratch_bytes() long
 * (2 x 128 floats per atom: the masses of mid-size footprints, written and read
 * within the call); its contents need no initialization. Any of
 * weight_dev / hi / lo may be NULL; hi+lo is the two-term TF32 split consumed by
 * tcst_gemm_tf32x3. */
int64_t tcst_weight_scratch_bytes(int64_t atoms, const tcst_axis *out_axis,
                                  const tcst_axis *in_axis);
int tcst_assemble_weight(const void *atom_table_dev, int64_t atoms,
                         const tcst_axis *out_axis, const tcst_axis *in_axis,
                         void *scratch_dev, int64_t scratch_bytes, float *weight_dev,
                         int64_t ld_weight, float *weight_hi_dev, float *weight_lo_dev,
                         int64_t ld_split, void *stream);

/* Weight assembly for the f16 three-product GEMM: W (float32, required) as
 * tcst_assemble_weight, max |W| folded into *amax_dev (start it at 0) while the
 * tiles are written, then the f16 split of tcst_split_f16 into hi/lo with its
 * power-of-two scale in *scale_dev. */
int tcst_assemble_weight_f16(const void *atom_table_dev, int64_t atoms,
                             const tcst_axis *out_axis, const tcst_axis *in_axis,
                             void *scratch_dev, int64_t scratch_bytes, float *weight_dev,
                             int64_t ld_weight, float *amax_dev, void *hi_dev, void *lo_dev,
                             int64_t ld_split, float *scale_dev, void *stream);

/* A window W[row0 : row0 + rows, col0 : col0 + cols] of the same weight
 * (row0 and col0 multiples of 32; W[r][c] stored at (r - row0, c - col0)),
 * with its own max |W| and f16 split: the output-row band (and input-column
 * band) of one rank when a layer is sharded by output rows. No counterpart in
 * the reference (its layer is not sharded). Values equal the full assembly's
 * bit for bit. */
int tcst_assemble_weight_window_f16(const void *atom_table_dev, int64_t atoms,
                                    const tcst_axis *out_axis, const tcst_axis *in_axis,
                                    void *scratch_dev, int64_t scratch_bytes, int64_t row0,
                                    int64_t rows, int64_t col0, int64_t cols, float *weight_dev,
                                    int64_t ld_weight, float *amax_dev, void *hi_dev,
                                    void *lo_dev, int64_t ld_split, float *scale_dev,
                                    void *stream);

/* No counterpart in the reference. The same weight assembly as
 * tcst_assemble_weight for callers that cannot allocate device memory (a plugin
 * inside a host framework whose allocator owns the device, or a fixed-footprint
 * deployment): the scratch is a fixed array built into this library,
 * tcst_static_weight_scratch_bytes() = 32 MiB, which every GPU that loads the
 * library holds until exit. That covers up to 32,768 atoms (1 KiB each); a
 * layer whose tcst_weight_scratch_bytes() exceeds it is rejected with
 * TCST_ERR_UNSUPPORTED. The first call on a device looks up the array's device
 * address; make that first call before any stream capture. Every call shares
 * the one array; calls that overlap on the GPU (same device, different streams)
 * race. Nothing is allocated. */
int tcst_assemble_weight_static(const void *atom_table_dev, int64_t atoms,
                                const tcst_axis *out_axis, const tcst_axis *in_axis,
                                float *weight_dev, int64_t ld_weight, float *weight_hi_dev,
                                float *weight_lo_dev, int64_t ld_split, void *stream);
int64_t tcst_static_weight_scratch_bytes(void);

/* Two-term TF32 split: hi = rn_tf32(x), lo = rn_tf32(x - hi). */
int tcst_split_tf32(const float *x_dev, int64_t rows, int64_t cols, int64_t ld_x,
                    float *hi_dev, float *lo_dev, int64_t ld_out, void *stream);

/* C[s][m][n] = sum_{k in split s} A[m,k] B[n,k] on tcgen05 tensor cores with the
 * three-product TF32 split (hi*hi + hi*lo + lo*hi, float32 accumulation in TMEM).
 * A is K-major (a[m*lda+k]) or, with a_mn_major, MN-major (a[k*lda+m]); B alike.
 * Leading dimensions must be multiples of 4 and bases 16-byte aligned.
 * Stands in for the float32 GEMMs of _backends/torch/operators/linear.py:59-65
 * and their autograd backward. */
int tcst_gemm_tf32x3(int64_t M, int64_t N, int64_t K,
                     const float *a_hi_dev, const float *a_lo_dev, int64_t lda, int32_t a_mn_major,
                     const float *b_hi_dev, const float *b_lo_dev, int64_t ldb, int32_t b_mn_major,
                     float *c_dev, int64_t ldc, int32_t split_k, int64_t split_stride,
                     uint32_t *status_dev, void *stream);

/* The same three-product contraction on f16 split planes (kind::f16 at twice
 * the TF32 rate, half the operand bytes). Planes come from tcst_split_f16
 * (element type IEEE half, leading dimensions multiples of 8); a_scale_dev /
 * b_scale_dev point at the per-tensor power-of-two scales that split stored,
 * and the epilogue multiplies by 1 / (s_A s_B) (exact). Otherwise as
 * tcst_gemm_tf32x3. */
int tcst_gemm_f16x3(int64_t M, int64_t N, int64_t K, const void *a_hi_dev, const void *a_lo_dev,
                    int64_t lda, int32_t a_mn_major, const float *a_scale_dev,
                    const void *b_hi_dev, const void *b_lo_dev, int64_t ldb,
                    int32_t b_mn_major, const float *b_scale_dev, float *c_dev, int64_t ldc,
                    int32_t split_k, int64_t split_stride, uint32_t *status_dev, void *stream);

/* Y = X W^T as tcst_gemm_f16x3 with both operands K-major and no split,
 * followed in the epilogue by the MSE gradient of a training step (the
 * driver-side loss of the reference's examples): writes dY = (Y - T) * scale
 * to dy_dev (Y itself is not stored), one double sum of (Y - T)^2 per 32 output
 * rows of a 128 x 256 tile to loss_partial_dev (*partials of them, fixed
 * order), and folds max |dY| into *amax_dev (nullable) for the f16 split of
 * dY. K must be positive. */
int tcst_gemm_f16x3_mse(int64_t M, int64_t N, int64_t K, const void *a_hi_dev,
                        const void *a_lo_dev, int64_t lda, const float *a_scale_dev,
                        const void *b_hi_dev, const void *b_lo_dev, int64_t ldb,
                        const float *b_scale_dev, const float *target_dev, int64_t ld_target,
                        float scale, float *dy_dev, int64_t ld_dy, double *loss_partial_dev,
                        int32_t *partials, float *amax_dev, uint32_t *status_dev, void *stream);

/* *amax_dev = max(*amax_dev, max |x|) over a [rows][cols] float32 view (start
 * it at 0). */
int tcst_absmax(const float *x_dev, int64_t rows, int64_t cols, int64_t ld, float *amax_dev,
                void *stream);

/* F16 split for tcst_gemm_f16x3: s = 2^k with max |s x| in [2^14, 2^15) from
 * *amax_dev (s = 1 when it is 0 or not finite), hi = rn_f16(s x),
 * lo = rn_f16(s x - hi); s is stored in *scale_dev. */
int tcst_split_f16(const float *x_dev, int64_t rows, int64_t cols, int64_t ld_x,
                   const float *amax_dev, void *hi_dev, void *lo_dev, int64_t ld_out,
                   float *scale_dev, void *stream);

/* MSE upstream gradient in float32: dY = (Y - T) * scale (dy_dev may equal y_dev
 * with ld_out == ld), per-block sums of (Y - T)^2 as tcst_mse_grad, and
 * max |dY| folded into *amax_dev (nullable) for the f16 split. */
int tcst_mse_grad_f32(const float *y_dev, const float *target_dev, int64_t rows, int64_t cols,
                      int64_t ld, float scale, float *dy_dev, int64_t ld_out,
                      double *loss_partial_dev, int32_t *blocks, float *amax_dev, void *stream);

/* Atom-parameter gradient from G = sum_s G_s = dY^T X ([N_out][ldg] per split):
 * d amp, d mu_out, d mu_in and d R reduced over each atom footprint in a fixed
 * order, then the rational (a, q) or Polar (s, t) chain. Replaces the autograd
 * backward of radius_cell_mass.factors through integrated_cells,
 * density_coefficients and physical_parameters. grad_dev is [atoms][4].
 * With split > 1 the partials are first summed in place into G_0 (the other
 * partials are left as they were). */
int tcst_pullback(const void *atom_table_dev, int64_t atoms, const tcst_axis *out_axis,
                  const tcst_axis *in_axis, float *g_dev, int64_t ldg,
                  int32_t split, int64_t split_stride, float *grad_dev, void *stream);

/* tcst_pullback over the chart rows [row0, row0 + rows) of G only (g_dev holds
 * those rows, row0 first; split partials as tcst_pullback): every atom gets
 * the part of its gradient that its footprint rows inside the band
 * contribute, atoms outside the band get zero. Summed over a partition of the
 * rows this is tcst_pullback's gradient (up to float32 summation order): the
 * halo-atom reduction of a layer sharded by output rows. */
int tcst_pullback_band(const void *atom_table_dev, int64_t atoms, const tcst_axis *out_axis,
                       const tcst_axis *in_axis, float *g_dev, int64_t ldg, int32_t split,
                       int64_t split_stride, int64_t row0, int64_t rows, float *grad_dev,
                       void *stream);

/* Fused CSTAdamW step on [atoms][4] rows, in place: AdamW moments and proposal,
 * field_lrs rescale, then the rational projection
 * (_backends/torch/updates/rational_radius.py:10-29) or the Polar activity law
 * with torus retraction (_backends/torch/algorithms/polar_update/executor.py:42-112,
 * _backends/torch/geometry/flat_torus.py:30-35) and, when amplitude_decay is
 * nonzero, the Polar amplitude decay (executor.py:18-41). A nonzero
 * amplitude_decay with kind TCST_RATIONAL is an argument error, as the reference
 * rejects amplitude decay for non-Polar atoms (operators/atom_update.py:42-66). */
int tcst_optimizer_step(float *p_dev, const float *grad_dev, float *exp_avg_dev,
                        float *exp_avg_sq_dev, int64_t atoms, int32_t kind,
                        const tcst_adamw *params, void *stream);

/* The coordinate law alone, for an optimizer that computed its own AdamW
 * proposal and field rescale: proposal_dev ([atoms][4], in place) becomes the
 * rational projection or the Polar activity law with torus retraction and
 * amplitude decay, applied from previous_dev ([atoms][4], the point before the
 * step; must not alias the proposal). Only the coordinate-law fields of params
 * are read (amplitude_cap, polar_*, period_out/in, amplitude_decay). Replaces
 * the torch atom_update Algorithm's execute
 * (_backends/torch/algorithms/atom_update/algorithm.py:58-83:
 * apply_parameter_update, then decay_amplitude). */
int tcst_coordinate_update(float *proposal_dev, const float *previous_dev, int64_t atoms,
                           int32_t kind, const tcst_adamw *params, void *stream);

/* The same step with the tcst_adamw scalars in device memory (16-byte aligned),
 * read when the kernel runs, so a captured CUDA graph can replay the step while
 * the host refreshes the bias corrections between replays. No reference
 * counterpart: the reference's optimizer reads its scalars on the host. */
int tcst_optimizer_step_device(float *p_dev, const float *grad_dev, float *exp_avg_dev,
                               float *exp_avg_sq_dev, int64_t atoms, int32_t kind,
                               const tcst_adamw *params_dev, void *stream);

/* Per-step optimizer scalars without a host-to-device copy in front of a
 * captured step: a ring of `slots` slots in pinned (device-mapped) host memory,
 * `slot_bytes` apart (a multiple of 16, at least TCST_RING_SLOT_MIN), each a
 * tcst_adamw at offset 0 and a uint32 sequence number at TCST_RING_SEQ_OFFSET.
 * tcst_scalar_ring_fetch (one CTA) copies slot c % slots into the device state
 * block (TCST_RING_STATE_BYTES, 16-byte aligned, zero before the first fetch;
 * word 0 is the use count c, advanced by one per fetch), marking it valid when
 * the slot's sequence number is c and raising TCST_STATUS_SEQUENCE in
 * status_dev when it is not. tcst_optimizer_step_ring is
 * tcst_optimizer_step with the scalars of the state block, and leaves p,
 * exp_avg and exp_avg_sq unchanged when the block is not valid. The host
 * writes slot c before enqueuing fetch c and may rewrite it once that fetch
 * has run. No reference counterpart (see tcst_optimizer_step_device). */
#define TCST_RING_SEQ_OFFSET ((sizeof(tcst_adamw) + 15) / 16 * 16)
#define TCST_RING_SLOT_MIN (TCST_RING_SEQ_OFFSET + 16)
#define TCST_RING_STATE_BYTES (16 + TCST_RING_SEQ_OFFSET)
int tcst_scalar_ring_fetch(const void *ring_host, int32_t slots, int64_t slot_bytes,
                           void *ring_state_dev, uint32_t *status_dev, void *stream);
int tcst_optimizer_step_ring(float *p_dev, const float *grad_dev, float *exp_avg_dev,
                             float *exp_avg_sq_dev, int64_t atoms, int32_t kind,
                             const void *ring_state_dev, void *stream);

/* MSE upstream gradient dY = (Y - T) * scale split into TF32 hi/lo planes, plus
 * per-block partial sums of (Y - T)^2 in loss_partial_dev[blocks] (double).
 * Returns the number of partial blocks through *blocks (nullable). */
int tcst_mse_grad(const float *y_dev, const float *target_dev, int64_t rows, int64_t cols,
                  int64_t ld, float scale, float *dy_hi_dev, float *dy_lo_dev,
                  int64_t ld_out, double *loss_partial_dev, int32_t *blocks, void *stream);

/* Per-atom Frobenius energy amp^2 |m_out|^2 |m_in|^2 (images folded), used by
 * the variance-matching initializer (_backends/torch/initialization.py:52-83). */
int tcst_atom_energies(const void *atom_table_dev, int64_t atoms, const tcst_axis *out_axis,
                       const tcst_axis *in_axis, double *energy_dev, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TCST_B200_H */
