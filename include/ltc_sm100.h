/*
 * ltc_sm100.h -- C-ABI of the B200 (sm_100a) LTC ODE-solver library (libltc_sm100.so).
 *
 * The library replaces the reference's compiled solver, the pybind11 module
 * built from csrc/ltc_kernels.cu (bindings at csrc/ltc_kernels.cu:1307-1314),
 * which ltc_cuda.py loads and calls from LTCCudaForward (ltc_cuda.py:241-359).
 * All pointers are DEVICE pointers to contiguous fp32 arrays unless stated;
 * every call is asynchronous on the given stream and allocates nothing: the
 * caller provides the output, saved-state and workspace buffers whose sizes
 * ltc_plan() reports.  Status 0 = success; non-zero = error, described by
 * ltc_last_error() (per calling thread).
 *
 * Layouts:  x (B,T,D); state (B,H); outputs (B,T,H);
 *           recurrent matrices (H,H) indexed [presynaptic, postsynaptic];
 *           sensory matrices (D,H) indexed [input, postsynaptic]; vectors (H).
 */
#ifndef LTC_SM100_H
#define LTC_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ltc_stream_t; /* == cudaStream_t */

/* Problem size.  ode_unfolds and epsilon mean what they mean in
 * ltc_full_forward (csrc/ltc_kernels.cu:1179-1181). */
typedef struct {
  int32_t B, T, D, H;
  int32_t ode_unfolds;
  float epsilon;
  int32_t flags; /* LTC_FLAG_* */
} LtcDims;

#define LTC_FLAG_FORCE_WIDE 1 /* use the streamed wide-H kernels even for H <= 64 */
/* Memory-lean training (the reference keeps every unfold's state: v_buffers
 * (T,U,B,H), csrc/ltc_kernels.cu:1205-1212).  The forward saves only the state
 * at each step boundary ((T+1)*B*H floats instead of (2*T*U+1)*B*H); the
 * backward recomputes the unfolds segment by segment (lean_chunk_steps steps per
 * segment, newest first) with the forward kernels and accumulates the parameter
 * partials across segments.  Cost: one extra recurrent + sensory forward. */
#define LTC_FLAG_LEAN_SAVE 2
/* Skip structurally-zero recurrent synapses (no counterpart in the reference, whose
 * kernels visit all H*H synapses, csrc/ltc_kernels.cu:115-192,549-668).  A synapse
 * whose w_pos and w_erev are both zero adds nothing to the forward solve and has
 * dL/dz = 0, so its only gradient terms are those of w_pos / w_erev at its own
 * position.  With this flag the caller declares those entries unused -- true
 * whenever w_pos = softplus(w) * mask, since the chain rule multiplies them by the
 * mask -- and the solver visits only the nonzero synapses; the four recurrent
 * gradients (w_pos, w_erev, mu, sigma) are written as zero at the skipped
 * positions.  Every other output is unchanged.  Honoured for H <= 64 and for
 * 128 < H <= 512 (64 < H <= 128 runs the dense kernels); the synapse tables are
 * rebuilt on the device at every call.  Capacity: for 32 < H <= 64 every neuron may
 * have at most 48 nonzero incoming and 48 nonzero outgoing synapses (any pattern
 * fits for H <= 32); for 128 < H <= 512 (HP = 256 for H <= 256, else 512) at most
 * 8192 nonzero synapses enter each block of HP/8 consecutive neurons, and inside
 * each such block of rows, ranked by outgoing count and paired c-th heaviest with
 * c-th lightest in groups of 4 pairs, 4*ceil(max ceil(heavy/8)/4) +
 * 4*ceil(max ceil(light/8)/4) <= 32 (the rule ltc_cuda.skip_zero_synapses_fits
 * applies; roughly 120 per row at uniform density).  The library cannot
 * report a violation without a device sync, so a call that exceeds it writes NaN
 * to its outputs and gradients; check the pattern before setting the flag.
 * The same flag makes the sensory forward visit only the sensory synapses with
 * sensory_w_pos != 0 (any pattern; D up to 682, larger D keeps the dense pass); that changes no output
 * beyond summation order and no gradient. */
#define LTC_FLAG_SKIP_ZERO_SYNAPSES 4
/* Also skip the zero sensory synapses (sensory_w_pos == 0) in the sensory backward
 * (no counterpart in the reference, csrc/ltc_kernels.cu:675-950 visits all D*H).
 * Like the recurrent case, the caller declares the sensory_w_pos gradient unused at
 * those positions (true for softplus(w) * mask); the four sensory gradients are
 * written as zero there.  Honoured together with LTC_FLAG_SKIP_ZERO_SYNAPSES, for
 * any H, unless LTC_FLAG_FORCE_WIDE is set.  Capacity (H > 32):
 * within each block of 64 consecutive inputs x 64 consecutive columns every input
 * may feed at most 48 nonzero synapses and every column receive at most 48; beyond
 * it the outputs are NaN. */
#define LTC_FLAG_SKIP_ZERO_SENSORY (1 << 24)
/* Bits 8..23 of flags, if nonzero, fix the lean segment length in steps
 * (otherwise it is sized for about 512 MiB of per-unfold state). */
#define LTC_LEAN_CHUNK_SHIFT 8

/* The 11 parameter inputs of ltc_full_forward (csrc/ltc_kernels.cu:1167-1178),
 * untransposed, in the same order. */
typedef struct {
  const float* w_pos;         /* (H,H) softplus(w) * mask            */
  const float* w_erev;        /* (H,H) w_pos * erev                  */
  const float* mu;            /* (H,H)                               */
  const float* sigma;         /* (H,H)                               */
  const float* sensory_mu;    /* (D,H)                               */
  const float* sensory_sigma; /* (D,H)                               */
  const float* sensory_erev;  /* (D,H)                               */
  const float* sensory_w_pos; /* (D,H) softplus(sensory_w) * mask    */
  const float* cm_t;          /* (H)   softplus(cm) / (dt / unfolds) */
  const float* gleak_pos;     /* (H)                                 */
  const float* vleak;         /* (H)                                 */
} LtcParams;

/* The 13 gradient outputs of ltc_full_backward (csrc/ltc_kernels.cu:1139-1153 and
 * ltc_cuda.py:342-355), in the same order.  Every pointer must be valid. */
typedef struct {
  float* x_seq;          /* (B,T,D) */
  float* state;          /* (B,H)   */
  float* w_pos;          /* (H,H)   */
  float* w_erev;         /* (H,H)   */
  float* mu;             /* (H,H)   */
  float* sigma;          /* (H,H)   */
  float* sensory_mu;     /* (D,H)   */
  float* sensory_sigma;  /* (D,H)   */
  float* sensory_erev;   /* (D,H)   */
  float* sensory_w_pos;  /* (D,H)   */
  float* cm_t;           /* (H)     */
  float* gleak_pos;      /* (H)     */
  float* vleak;          /* (H)     */
} LtcGrads;

/* Buffer sizes (bytes) for a problem on the CURRENT device.  saved_bytes is the
 * forward state kept for the backward pass (replaces v_buffers_stacked and the
 * sensory stacks of ltc_full_forward, csrc/ltc_kernels.cu:1205-1212). */
typedef struct {
  size_t saved_bytes;
  size_t fwd_workspace_bytes;
  size_t bwd_workspace_bytes;
  int32_t wide;       /* 1 if the wide-H kernels will run */
  int32_t padded_h;   /* neuron count the kernels pad H to */
  int32_t fwd_ctas, bwd_ctas;
  int32_t lean_chunk_steps; /* steps per recomputed segment (LTC_FLAG_LEAN_SAVE), else 0 */
} LtcPlan;

int ltc_plan(const LtcDims* dims, LtcPlan* out);

/* Forward solve over all T steps (replaces ltc_full_forward,
 * csrc/ltc_kernels.cu:1165-1300).  h0 may be NULL (zero state).  saved may be
 * NULL when no backward pass follows (save_intermediates = false); otherwise it
 * must hold plan.saved_bytes. */
int ltc_forward(const LtcDims* dims, const LtcParams* params, const float* x, const float* h0,
                float* outputs, float* h_final, void* saved, void* workspace, size_t workspace_bytes,
                ltc_stream_t stream);

/* Backward pass over all T steps (replaces ltc_full_backward,
 * csrc/ltc_kernels.cu:962-1154).  grad_outputs is addressed with the element
 * strides go_strides[3] (B,T,H order; stride 0 allowed, e.g. from out.sum()).
 * grad_state may be NULL (no gradient on the returned state).  Deterministic:
 * no atomics; fixed-order reductions. */
int ltc_backward(const LtcDims* dims, const LtcParams* params, const float* x, const void* saved,
                 const float* grad_outputs, const int64_t go_strides[3], const float* grad_state,
                 const LtcGrads* grads, void* workspace, size_t workspace_bytes, ltc_stream_t stream);

/* Step-level calls for callers that drive the time loop themselves; they replace the
 * reference's per-step exports (csrc/ltc_kernels.cu:675-950, bound at :1308-1311).
 * dims: B, H (and D for the sensory calls, ode_unfolds/epsilon for the unfold calls);
 * T is ignored (one step).  Matrices untransposed as in LtcParams (only the fields
 * a call uses must be set).  Each call needs a workspace of
 * ltc_step_workspace_bytes(dims, kind) bytes, kind = 0 sensory forward, 1 unfold
 * forward, 2 sensory backward, 3 unfold backward. */
int ltc_step_workspace_bytes(const LtcDims* dims, int kind, size_t* bytes);
/* ltc_sensory_fwd (csrc/ltc_kernels.cu:675): inputs (B,D) -> w_num, w_den (B,H). */
int ltc_step_sensory_forward(const LtcDims* dims, const LtcParams* params, const float* inputs, float* w_num,
                             float* w_den, void* workspace, size_t workspace_bytes, ltc_stream_t stream);
/* ltc_ode_unfold_fwd (csrc/ltc_kernels.cu:716): ode_unfolds implicit-Euler unfolds from
 * state (B,H) with the step's sensory sums; v_buffer (ode_unfolds,B,H), the input of
 * every unfold, may be NULL. */
int ltc_step_unfold_forward(const LtcDims* dims, const LtcParams* params, const float* state, const float* w_num,
                            const float* w_den, float* state_out, float* v_buffer, void* workspace,
                            size_t workspace_bytes, ltc_stream_t stream);
/* ltc_sensory_bwd (csrc/ltc_kernels.cu:780): gradients of the sensory sums -> grad of
 * inputs (B,D) and of sensory sigma, mu, w_pos, erev (D,H). */
int ltc_step_sensory_backward(const LtcDims* dims, const LtcParams* params, const float* grad_w_num,
                              const float* grad_w_den, const float* inputs, float* grad_inputs, float* g_sigma,
                              float* g_mu, float* g_w_pos, float* g_erev, void* workspace, size_t workspace_bytes,
                              ltc_stream_t stream);
/* ltc_ode_unfold_bwd (csrc/ltc_kernels.cu:845): from v_buffer (ode_unfolds,B,H) and
 * dL/d(final state) (B,H) -> dL/d(initial state), dL/d(w_num, w_den) (B,H) and the
 * recurrent-parameter gradients.  The step's unfolds are recomputed from v_buffer[0]. */
int ltc_step_unfold_backward(const LtcDims* dims, const LtcParams* params, const float* v_buffer, const float* w_num,
                             const float* w_den, const float* grad_output, float* grad_v, float* grad_w_num,
                             float* grad_w_den, float* g_w_pos, float* g_w_erev, float* g_mu, float* g_sigma,
                             float* g_cm, float* g_gleak, float* g_vleak, void* workspace, size_t workspace_bytes,
                             ltc_stream_t stream);

/* Module preamble, fused (replaces the PyTorch ops of ltc.py:259 and ltc.py:266):
 *   y = (LayerNorm(x) * ln_w + ln_b) * in_w + in_b     over the last dim D <= 1024,
 * biased variance, eps as nn.LayerNorm.  x, y: (rows, D); stats: (rows, 2) =
 * (mean, 1/sqrt(var+eps)) kept for the backward.  The backward writes dx and the
 * four (D) parameter gradients (deterministic, fixed-order reductions) and needs
 * a workspace of ltc_preamble_workspace_bytes(rows, D) bytes. */
int ltc_preamble_forward(int64_t rows, int32_t D, float eps, const float* x, const float* ln_w,
                         const float* ln_b, const float* in_w, const float* in_b, float* y, float* stats,
                         ltc_stream_t stream);
size_t ltc_preamble_workspace_bytes(int64_t rows, int32_t D);
int ltc_preamble_backward(int64_t rows, int32_t D, const float* x, const float* dy, const float* ln_w,
                          const float* ln_b, const float* in_w, const float* stats, float* dx, float* g_ln_w,
                          float* g_ln_b, float* g_in_w, float* g_in_b, void* workspace, size_t workspace_bytes,
                          ltc_stream_t stream);

/* Size of the fixed device scratch array behind ltc_forward_noalloc (16 MiB per GPU). */
#define LTC_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/* Forward solve that allocates nothing and takes no workspace (no counterpart in
 * the reference).  For callers that may not allocate GPU memory where they run
 * the solver -- hosts that own every allocation (a plugin in a serving runtime
 * with a fixed memory budget) or latency-critical loops in which cudaMalloc
 * would synchronise the device.  Same inputs and outputs as ltc_forward with
 * saved == NULL.  Its scratch is one static __device__ array of
 * LTC_NOALLOC_SCRATCH_BYTES per GPU, held until exit; problems that need more
 * are rejected with an error.  The first call on a device resolves the array's
 * address (cudaGetSymbolAddress): make it before any stream capture.  All calls
 * on a device share the array, so calls that overlap on the GPU race: serialise
 * them.  Its launches create no timing events: they are not counted by
 * ltc_launch_count() nor timed by ltc_timing_enable(). */
int ltc_forward_noalloc(const LtcDims* dims, const LtcParams* params, const float* x, const float* h0,
                        float* outputs, float* h_final, ltc_stream_t stream);

/* Kernel identifiers of the launches each call issues (forward: PACK_FWD,
 * SENSORY_FWD, RECURRENT_FWD; backward: PACK_BWD, RECURRENT_BWD, SENSORY_BWD, FINISH; the fused
 * module preamble: PREAMBLE_FWD, PREAMBLE_BWD). */
enum {
  LTC_KERNEL_PACK_FWD = 0,
  LTC_KERNEL_SENSORY_FWD = 1,
  LTC_KERNEL_RECURRENT_FWD = 2,
  LTC_KERNEL_PACK_BWD = 3,
  LTC_KERNEL_RECURRENT_BWD = 4,
  LTC_KERNEL_SENSORY_BWD = 5,
  LTC_KERNEL_FINISH = 6,
  LTC_KERNEL_PREAMBLE_FWD = 7,
  LTC_KERNEL_PREAMBLE_BWD = 8,
  LTC_NUM_KERNELS = 9
};

/* Per-launch device timing, process-wide (no counterpart in the
 * reference, whose bench times with torch.profiler, bench_ltc.py:292-387).
 * While enabled, every launch is bracketed by a cudaEvent pair recorded on its
 * own stream.  ltc_timing_collect() waits for them, writes the summed
 * milliseconds and launch counts per LTC_KERNEL_* id (n >= LTC_NUM_KERNELS) and
 * clears the record. */
int ltc_timing_enable(int on);
int ltc_timing_collect(double* total_ms, int32_t* launches, int n);

/* Number of kernels launched through the library by this process (every entry
 * point except ltc_forward_noalloc). */
int64_t ltc_launch_count(void);

/* Number of bounded in-kernel waits (the per-unfold exchange between the CTAs
 * of a cluster, H in 65..128) that expired on the current device since the
 * library was loaded; 0 in a healthy process.  Synchronises with the device.
 * Returns -1 on a CUDA error. */
int ltc_wait_timeouts(void);

/* Checked build (no counterpart in the reference).  libltc_sm100_checked.so is the
 * same library compiled with -DLTC_CHECKED: the kernels test the indices of their
 * table-driven gathers, shared-memory slabs and output writes, and an index out of
 * its bound is counted and its access skipped instead of faulting the GPU.
 * ltc_checked_build() is the number of source files whose kernels carry checks in
 * that build, 0 in the normal one;
 * ltc_check_errors() synchronises the device, returns the number of failed checks
 * since the last call and the id of the first failing site (0 if none; the site ids
 * are the LTC_CHECK call sites in the sources), and resets them.  Returns 0, or -1
 * on a CUDA error. */
int ltc_checked_build(void);
int ltc_check_errors(int* count, int* first_site);

/* Last error message of the calling thread ("" if none). */
const char* ltc_last_error(void);

/* Library version (major*10000 + minor*100 + patch). */
int ltc_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LTC_SM100_H */
