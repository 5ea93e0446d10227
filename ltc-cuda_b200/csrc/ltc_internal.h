// Internal launch interfaces shared by the kernel translation units and the C-ABI layer.
#pragma once
#include <vector>

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ltc {
std::vector<int (*)(int*, int*)>& check_readers();

// ---- parameter packing --------------------------------------------------
struct PackArgs {
  const float* w_pos;   // (H,H)
  const float* w_erev;  // (H,H)
  const float* mu;      // (H,H)
  const float* sigma;   // (H,H)
  const float* smu;     // (D,H)
  const float* ssig;    // (D,H)
  const float* serev;   // (D,H)
  const float* sw;      // (D,H)
  const float* cm;      // (H)
  const float* gl;      // (H)
  const float* vl;      // (H)
  float4* pack;         // [HP][HP]  (sh, nh, w_pos, w_erev) indexed [p][q]
  float4* packT;        // [HP][HP]  same, indexed [q][p]   (may be null); see packT_qc
  int packT_qc;         // > 0: packT instead holds pack in rows [p] with each qc-column chunk
                        //      reordered from (ql, j) = (c/8, c%8) to (j, ql): the streamed
                        //      backward's TMA staging layout (qc = its chunk width)
  float4* spack;        // [D][HP]   (sh, nh, sw, sw*serev)
  float4* nrn;          // [HP]      (cm, gl, vl, gl*vl)
  int D, H, HP;
};
cudaError_t launch_pack(const PackArgs& a, cudaStream_t st);

// ---- sensory forward: sn/sd per row (row = b*T + t) ----------------------
struct SensFwdArgs {
  const float4* spack;  // [D][HP]
  const float* x;       // (rows, D)
  float* sn;            // (rows, H)
  float* sd;            // (rows, H)
  long long rows;
  int D, H, HP;
};
cudaError_t launch_sensory_fwd(const SensFwdArgs& a, int num_sms, cudaStream_t st);
// masked sensory synapses skipped (ltc_sensory_sparse.cu): per-column lists of the
// nonzero inputs, built on the device after the pack (sens_tables_bytes of workspace)
size_t sens_tables_bytes(int D, int HP);
bool sens_sparse_fits(int D);
cudaError_t launch_build_sens(const PackArgs& pa, void* tables, cudaStream_t st);
cudaError_t launch_sensory_fwd_sparse(const SensFwdArgs& a, const void* tables, int num_sms, cudaStream_t st);

// ---- sensory backward ----------------------------------------------------
struct SensBwdArgs {
  const float4* spack;  // [D][HP]
  const float* x;       // (rows, D)
  const float* gsn;     // (rows, H)
  const float* gsd;     // (rows, H)
  float* dx;            // (rows, D)   (nqc == 1) or dx partials [nqc][rows][D]
  float* part;          // [nsplit][4][D][HP] synapse partials (A_n, A_d, DZ, DZX)
  long long rows;
  int D, H, HP;
  int nsplit;           // row splits (gridDim.y)
};
struct SensBwdPlan {
  int qc;          // columns per CTA
  int nqc;         // column chunks
  int dpc;         // inputs d per CTA
  int ndc;         // d chunks
  int nsplit;      // row splits
  size_t part_floats;
  size_t dxpart_floats;  // 0 when nqc == 1
};
SensBwdPlan plan_sensory_bwd(long long rows, int D, int HP, int num_sms);
// tanh_space: the sensory partials are sums of a'*tanh and the finish kernel adds the
// column sums of g_sn, g_sd taken from the recurrent per-neuron partials (rows 3, 4)
cudaError_t launch_sensory_bwd(const SensBwdArgs& a, const SensBwdPlan& p, float* dxpart, bool tanh_space,
                               cudaStream_t st);
// masked sensory synapses skipped in the backward (LTC_FLAG_SKIP_ZERO_SENSORY, any
// skipping recurrent path; ltc_recurrent_sparse.cu): slot tables per 64 x 64 block
// (32 x 32 for H <= 32) of the sensory pattern, tanh space
size_t sens_bwd_tables_bytes(int D, int H, int HP);
void plan_sensory_bwd_sparse(SensBwdPlan& p, long long rows, int D, int H, int HP, int num_sms);
cudaError_t launch_build_sens_slots(const PackArgs& pa, void* tables, cudaStream_t st);
cudaError_t launch_sensory_bwd_sparse(const SensBwdArgs& a, const SensBwdPlan& p, const void* tables,
                                      float* dxpart, cudaStream_t st);

// ---- recurrent forward / backward ----------------------------------------
struct RecFwdArgs {
  const float4* pack;   // [HP][HP]
  const float4* nrn;    // [HP]
  const float* sn;      // (B*T, H)
  const float* sd;      // (B*T, H)
  const float* h0;      // (B,H) or null (zeros)
  float* out;           // (B,T,H) or null (recomputation for a lean backward)
  float* hT;            // (B,H) or null
  float* V;             // (T*U+1, B, H) or null
  float* R;             // (T*U, B, H) or null
  int B, T, H, U, HP;
  int ns;               // samples per CTA
  float eps;
  float* scratch;       // plan.scratch_fwd floats (streamed path)
  const void* tables;   // slot tables (sparse path, launch_build_slots)
};
struct RecBwdArgs {
  const float4* pack;   // [HP][HP] (fast path)
  const float4* packT;  // [HP][HP] (wide path)
  const float4* nrn;
  const float* V;
  const float* R;
  const float* gout;    // strided (B,T,H)
  long long go_sb, go_st, go_sh;
  const float* gstate;  // (B,H) or null
  float* gsn;           // (B*T, H)
  float* gsd;           // (B*T, H)
  float* gh0;           // (B,H)
  float* part;          // [slots][4][HP*HP]  synapse partials, layout [p][q] (fast) / [q][p] (wide)
  float* partn;         // [slots][3 or 5][HP] (see RecPlan::tanh_space)
  int B, T, H, U, HP;
  int ns;
  float* scratch;       // plan.scratch_bwd floats (streamed path)
  int accumulate;       // add to part/partn (segments of a lean backward) instead of overwriting
  const void* tables;   // slot tables (sparse path, launch_build_slots)
};
struct RecPlan {
  bool wide;       // not the register-resident kernels (streamed or generic wide-H)
  bool streamed;   // cluster-streamed kernels (128 < H <= 512)
  bool tanh_space; // synapse partials hold sum a'*tanh (a' = -a/4); partn has 5 rows (+ sum a_n, sum a_d)
  bool sparse;     // zero synapses skipped (LTC_FLAG_SKIP_ZERO_SYNAPSES): slot-table kernels (H <= 64) or
                   // cluster list kernels (128 < H <= 512, with streamed set)
  size_t scratch_fwd, scratch_bwd;  // floats of path-specific global scratch
  int HP;          // padded neuron count
  int ns_fwd, grid_fwd, threads_fwd;
  size_t smem_fwd;
  int ns_bwd, grid_bwd, threads_bwd, slots_bwd;
  size_t smem_bwd;
};
// skip_zero: the caller set LTC_FLAG_SKIP_ZERO_SYNAPSES (honoured for H <= 64 without force_wide)
RecPlan plan_recurrent(int B, int H, int num_sms, int force_wide, bool skip_zero = false);
// sparse path (ltc_recurrent_sparse.cu): slot tables built on the device from the
// recurrent parameters (sparse_tables_bytes(HP) of workspace), then the kernels
size_t sparse_tables_bytes(int HP);
void plan_sparse(RecPlan& p, int B, int num_sms);
cudaError_t launch_build_slots(const PackArgs& pa, void* tables, cudaStream_t st);
cudaError_t launch_sparse_fwd(const RecFwdArgs& a, const RecPlan& p, const void* tables, cudaStream_t st);
cudaError_t launch_sparse_bwd(const RecBwdArgs& a, const RecPlan& p, const void* tables, cudaStream_t st);
// 128 < H <= 512 (ltc_recurrent_csparse.cu; reached through the calls above)
size_t csp_tables_bytes(int HP);
void plan_csparse(RecPlan& p, int B, int num_clusters);
cudaError_t launch_build_csp(const PackArgs& pa, void* tables, cudaStream_t st);
cudaError_t launch_csp_fwd(const RecFwdArgs& a, const RecPlan& p, const void* tables, cudaStream_t st);
cudaError_t launch_csp_bwd(const RecBwdArgs& a, const RecPlan& p, const void* tables, cudaStream_t st);
// chunk width of the streamed backward (256 threads, 8-CTA clusters), 0 on other paths
inline int stream_chunk_cols(const RecPlan& p) { return p.streamed ? 16384 / p.HP : 0; }
cudaError_t launch_recurrent_fwd(const RecFwdArgs& a, const RecPlan& p, cudaStream_t st);
cudaError_t launch_recurrent_bwd(const RecBwdArgs& a, const RecPlan& p, cudaStream_t st);
// bounded cluster waits that expired on the current device (ltc_recurrent.cu)
int read_wait_timeouts(int* count);
int read_stream_wait_timeouts(int* count);  // ltc_recurrent_stream.cu

// ---- deterministic reductions and final gradient transforms --------------
struct FinishArgs {
  const float* rec_part;   // [rslots][4][HP*HP]
  const float* rec_partn;  // [rslots][3 or 5][HP]
  int rslots;
  bool rec_transposed;     // partial layout [q][p]
  bool rec_tanh_space;     // S0/S1 are sums of a'*tanh (a' = -a/4), partn rows 3/4 = sums of a_n/a_d
  // sparse path: synapses with w_pos == w_erev == 0 were skipped; their four
  // gradients are written as zero (their partial-slab entries are never written)
  const float* skip_w_pos; const float* skip_w_erev;
  // sensory synapses with sw == 0 were skipped in the sensory backward: their four
  // gradients are written as zero
  const float* skip_sw;
  const float* sens_part;  // [nsplit][4][D*HP]
  int nsplit;
  const float* dxpart;     // [nqc][rows*D] or null
  int nqc;
  long long rows;
  // inputs needed by the transforms
  const float* mu; const float* sigma;
  const float* smu; const float* ssig; const float* serev; const float* sw;
  // outputs
  float* g_w_pos; float* g_w_erev; float* g_mu; float* g_sigma;
  float* g_smu; float* g_ssig; float* g_serev; float* g_sw;
  float* g_cm; float* g_gl; float* g_vl;
  float* g_x;
  int D, H, HP;
};
cudaError_t launch_finish(const FinishArgs& a, int num_sms, cudaStream_t st);

// ---- module preamble: LayerNorm + input affine ---------------------------
struct PreambleArgs {
  const float* x;       // (rows, D) raw input
  const float* dy;      // (rows, D) gradient of the preamble output (backward)
  const float* ln_w; const float* ln_b; const float* in_w; const float* in_b;  // (D)
  float* y;             // (rows, D) output (forward)
  float* dx;            // (rows, D) input gradient (backward)
  float* stats;         // (rows, 2) mean, rstd
  float* part;          // [blocks][4][D] column-gradient partials (backward)
  float* g_in_w; float* g_in_b; float* g_ln_w; float* g_ln_b;  // (D)
  long long rows;
  int D;
  float eps;
};
int preamble_blocks(long long rows, int num_sms);
cudaError_t launch_preamble_fwd(const PreambleArgs& a, int num_sms, cudaStream_t st);
cudaError_t launch_preamble_bwd(const PreambleArgs& a, int num_sms, cudaStream_t st);

// Error reporting shared by every extern "C" entry point (ltc_last_error()).
void set_last_error(const char* msg);

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }
inline int pad_neurons(int H) { return H <= 32 ? 32 : (H <= 64 ? 64 : (H <= 128 ? 128 : round_up(H, 32))); }

}  // namespace ltc
