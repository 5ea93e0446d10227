// extern "C" entry points of libltc_sm100.so (declared in include/ltc_sm100.h).
//
// Host-side orchestration is three (forward) / four (backward) launches on the
// caller's stream, independent of T and ode_unfolds:
//   forward : pack -> sensory_fwd (all B*T rows) -> recurrent_fwd (all T*U unfolds)
//   backward: pack -> recurrent_bwd -> sensory_bwd -> finish (reductions + transforms)
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/ltc_sm100.h"
#include "ltc_internal.h"

namespace ltc {
// readers of the checked build's per-file error words (empty in the normal build)
std::vector<int (*)(int*, int*)>& check_readers() {
  static std::vector<int (*)(int*, int*)> v;
  return v;
}
void register_check_reader(int (*reader)(int*, int*)) { check_readers().push_back(reader); }
}  // namespace ltc

using namespace ltc;

namespace {

thread_local std::string g_last_error;

int fail(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return 1;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail("%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Optional per-launch timing (ltc_timing_enable): a cudaEvent pair recorded on
// the launch stream around every kernel; ltc_timing_collect() sums them.
struct Timing {
  bool on = false;
  std::vector<cudaEvent_t> start, stop;
  std::vector<int> kid;
  size_t used = 0;
  long long launches = 0;
};
Timing g_tm;           // process-wide: the backward pass runs on autograd's worker thread
std::mutex g_tm_mu;

class TimedLaunch {
 public:
  TimedLaunch(int kid, cudaStream_t st) : st_(st), idx_(-1) {
    std::lock_guard<std::mutex> lk(g_tm_mu);
    ++g_tm.launches;
    if (!g_tm.on) return;
    if (g_tm.used == g_tm.start.size()) {
      cudaEvent_t a, b;
      if (cudaEventCreate(&a) != cudaSuccess) return;
      if (cudaEventCreate(&b) != cudaSuccess) { cudaEventDestroy(a); return; }
      g_tm.start.push_back(a);
      g_tm.stop.push_back(b);
      g_tm.kid.push_back(kid);
    }
    idx_ = (long long)g_tm.used++;
    g_tm.kid[idx_] = kid;
    cudaEventRecord(g_tm.start[idx_], st_);
  }
  ~TimedLaunch() {
    if (idx_ < 0) return;
    std::lock_guard<std::mutex> lk(g_tm_mu);
    cudaEventRecord(g_tm.stop[idx_], st_);
  }

 private:
  cudaStream_t st_;
  long long idx_;
};

struct DeviceInfo {
  int sms = 0;
  int major = 0;
};

DeviceInfo device_info(int* err) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    *err = cuda_fail(e == cudaSuccess ? cudaErrorInvalidDevice : e, "cudaGetDevice");
    return DeviceInfo{};
  }
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev].sms == 0) {
    int sms = 0, major = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess) {
      *err = cuda_fail(e, "cudaDeviceGetAttribute");
      return DeviceInfo{};
    }
    cache[dev].sms = sms;
    cache[dev].major = major;
  }
  *err = 0;
  return cache[dev];
}

// Carves 256-byte aligned sub-buffers out of one caller-provided allocation.
struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

struct Layout {
  RecPlan rp;
  SensBwdPlan sp;
  long long rows;
  size_t saved_floats_v, saved_floats_r;
  bool lean;  // LTC_FLAG_LEAN_SAVE: saved = step-boundary states; the backward recomputes segments
  bool skip_sens;  // LTC_FLAG_SKIP_ZERO_SYNAPSES: the sensory forward visits only sw != 0
  bool skip_sens_bwd;  // LTC_FLAG_SKIP_ZERO_SENSORY: so does the sensory backward (H <= 64)
  int tc;     // lean segment length in steps
};

int check_dims(const LtcDims* d) {
  if (!d) return fail("dims is NULL");
  if (d->B < 1 || d->T < 1 || d->D < 1 || d->H < 1 || d->ode_unfolds < 1)
    return fail("invalid dims: B=%d T=%d D=%d H=%d ode_unfolds=%d (all must be >= 1)", d->B, d->T, d->D,
                d->H, d->ode_unfolds);
  if (d->H > 512) return fail("H=%d exceeds the supported maximum of 512", d->H);
  return 0;
}

int make_layout(const LtcDims* d, Layout* L, DeviceInfo* di) {
  if (check_dims(d)) return 1;
  int err = 0;
  *di = device_info(&err);
  if (err) return 1;
  if (di->major != 10)
    return fail("libltc_sm100 requires an sm_100 (B200-class) GPU; current device is compute capability %d.x",
                di->major);
  L->rp = plan_recurrent(d->B, d->H, di->sms, d->flags & LTC_FLAG_FORCE_WIDE,
                         (d->flags & LTC_FLAG_SKIP_ZERO_SYNAPSES) != 0);
  L->rows = (long long)d->B * d->T;
  L->skip_sens = (d->flags & LTC_FLAG_SKIP_ZERO_SYNAPSES) && !(d->flags & LTC_FLAG_FORCE_WIDE) &&
                 sens_sparse_fits(d->D);
  L->sp = plan_sensory_bwd(L->rows, d->D, L->rp.HP, di->sms);
  // the sparse sensory backward works in tanh space: it needs the recurrent backward's
  // per-column adjoint sums, which every path but the forced wide one provides
  L->skip_sens_bwd = (d->flags & LTC_FLAG_SKIP_ZERO_SENSORY) && (d->flags & LTC_FLAG_SKIP_ZERO_SYNAPSES) &&
                     L->rp.tanh_space;
  if (L->skip_sens_bwd) plan_sensory_bwd_sparse(L->sp, L->rows, d->D, d->H, L->rp.HP, di->sms);
  const size_t tu = (size_t)d->T * d->ode_unfolds;
  L->lean = (d->flags & LTC_FLAG_LEAN_SAVE) != 0;
  L->tc = 0;
  if (L->lean) {
    // saved: h0 (B,H) + the step outputs (B,T,H), i.e. the state at every step boundary
    L->saved_floats_v = (size_t)(d->T + 1) * d->B * d->H;
    L->saved_floats_r = 0;
    const int fixed = (d->flags >> LTC_LEAN_CHUNK_SHIFT) & 0xFFFF;
    if (fixed > 0) {
      L->tc = fixed;
    } else {  // about 512 MiB of per-segment state (V, R, staged x and sensory sums)
      const double per_step =
          4.0 * ((2.0 * d->ode_unfolds + 4.0) * d->B * d->H + (double)d->B * d->D);
      const double n = (512.0 * 1024 * 1024) / per_step;
      L->tc = n < 1.0 ? 1 : (n > d->T ? d->T : (int)n);
    }
    if (L->tc > d->T) L->tc = d->T;
  } else {
    L->saved_floats_v = (tu + 1) * d->B * d->H;
    L->saved_floats_r = tu * d->B * d->H;
  }
  return 0;
}

struct FwdBuffers {
  float4 *pack, *spack, *nrn;
  float *sn, *sd, *scratch;
  void* tables;   // sparse path only
  void* stables;  // sensory lists (skip_sens only)
};
size_t carve_fwd(const LtcDims* d, const Layout& L, void* ws, FwdBuffers* b) {
  Carver c(ws);
  const int HP = L.rp.HP;
  b->pack = c.take<float4>((size_t)HP * HP);
  b->spack = c.take<float4>((size_t)d->D * HP);
  b->nrn = c.take<float4>(HP);
  b->sn = c.take<float>((size_t)L.rows * d->H);
  b->sd = c.take<float>((size_t)L.rows * d->H);
  b->scratch = L.rp.scratch_fwd ? c.take<float>(L.rp.scratch_fwd) : nullptr;
  b->tables = L.rp.sparse ? c.take<char>(sparse_tables_bytes(HP)) : nullptr;
  b->stables = L.skip_sens ? c.take<char>(sens_tables_bytes(d->D, HP)) : nullptr;
  return c.off + 256;
}

struct BwdBuffers {
  float4 *pack, *packT, *spack, *nrn;
  float *gsn, *gsd, *rpart, *rpartn, *spart, *dxpart, *scratch;
  // lean backward: one segment's staged inputs, recomputed state and outputs
  float *xc, *snc, *sdc, *gsnc, *gsdc, *Vc, *Rc, *hs, *ghA, *ghB, *fscratch;
  void* tables;   // sparse path only
  void* stables;  // sensory lists (lean recompute with skip_sens only)
  void* sbtables;  // sensory backward slot tables (skip_sens_bwd only)
};
size_t carve_bwd(const LtcDims* d, const Layout& L, void* ws, BwdBuffers* b) {
  Carver c(ws);
  const int HP = L.rp.HP;
  b->pack = c.take<float4>((size_t)HP * HP);
  b->packT = c.take<float4>((size_t)HP * HP);
  b->spack = c.take<float4>((size_t)d->D * HP);
  b->nrn = c.take<float4>(HP);
  b->gsn = c.take<float>((size_t)L.rows * d->H);
  b->gsd = c.take<float>((size_t)L.rows * d->H);
  b->rpart = c.take<float>((size_t)L.rp.slots_bwd * 4 * HP * HP);
  b->rpartn = c.take<float>((size_t)L.rp.slots_bwd * 5 * HP);
  b->spart = c.take<float>(L.sp.part_floats);
  b->dxpart = L.sp.dxpart_floats ? c.take<float>(L.sp.dxpart_floats) : nullptr;
  b->scratch = L.rp.scratch_bwd ? c.take<float>(L.rp.scratch_bwd) : nullptr;
  b->tables = L.rp.sparse ? c.take<char>(sparse_tables_bytes(HP)) : nullptr;
  b->stables = L.lean && L.skip_sens ? c.take<char>(sens_tables_bytes(d->D, HP)) : nullptr;
  b->sbtables = L.skip_sens_bwd ? c.take<char>(sens_bwd_tables_bytes(d->D, d->H, HP)) : nullptr;
  b->xc = b->snc = b->sdc = b->gsnc = b->gsdc = b->Vc = b->Rc = b->hs = b->ghA = b->ghB = b->fscratch = nullptr;
  if (L.lean) {
    const size_t BH = (size_t)d->B * d->H, tcu = (size_t)L.tc * d->ode_unfolds;
    b->xc = c.take<float>((size_t)d->B * L.tc * d->D);
    b->snc = c.take<float>(BH * L.tc);
    b->sdc = c.take<float>(BH * L.tc);
    b->gsnc = c.take<float>(BH * L.tc);
    b->gsdc = c.take<float>(BH * L.tc);
    b->Vc = c.take<float>((tcu + 1) * BH);
    b->Rc = c.take<float>(tcu * BH);
    b->hs = c.take<float>(BH);
    b->ghA = c.take<float>(BH);
    b->ghB = c.take<float>(BH);
    b->fscratch = L.rp.scratch_fwd ? c.take<float>(L.rp.scratch_fwd) : nullptr;
  }
  return c.off + 256;
}

PackArgs pack_args(const LtcDims* d, const LtcParams* p, int HP) {
  PackArgs a{};
  a.w_pos = p->w_pos; a.w_erev = p->w_erev; a.mu = p->mu; a.sigma = p->sigma;
  a.smu = p->sensory_mu; a.ssig = p->sensory_sigma; a.serev = p->sensory_erev; a.sw = p->sensory_w_pos;
  a.cm = p->cm_t; a.gl = p->gleak_pos; a.vl = p->vleak;
  a.D = d->D; a.H = d->H; a.HP = HP;
  return a;
}

int check_params(const LtcParams* p) {
  if (!p) return fail("params is NULL");
  const void* ptrs[] = {p->w_pos, p->w_erev, p->mu, p->sigma, p->sensory_mu, p->sensory_sigma,
                        p->sensory_erev, p->sensory_w_pos, p->cm_t, p->gleak_pos, p->vleak};
  for (const void* q : ptrs)
    if (!q) return fail("a parameter pointer is NULL");
  return 0;
}

int lean_recurrent_backward(const LtcDims* dims, const Layout& L, const DeviceInfo& di, const BwdBuffers& b,
                            const float* ck, const float* x, RecBwdArgs ra, cudaStream_t st);

}  // namespace

namespace ltc {
// Lets other translation units of the library report through ltc_last_error().
void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }
}  // namespace ltc

extern "C" {

const char* ltc_last_error(void) { return g_last_error.c_str(); }

int ltc_version(void) { return 100; }

int ltc_timing_enable(int on) {
  std::lock_guard<std::mutex> lk(g_tm_mu);
  g_tm.on = on != 0;
  g_tm.used = 0;
  return 0;
}

int ltc_timing_collect(double* total_ms, int32_t* launches, int n) {
  if (!total_ms || !launches || n < LTC_NUM_KERNELS) return fail("ltc_timing_collect: need %d slots", LTC_NUM_KERNELS);
  std::lock_guard<std::mutex> lk(g_tm_mu);
  for (int k = 0; k < n; ++k) {
    total_ms[k] = 0.0;
    launches[k] = 0;
  }
  for (size_t i = 0; i < g_tm.used; ++i) {
    cudaError_t e = cudaEventSynchronize(g_tm.stop[i]);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize");
    float ms = 0.f;
    e = cudaEventElapsedTime(&ms, g_tm.start[i], g_tm.stop[i]);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventElapsedTime");
    total_ms[g_tm.kid[i]] += ms;
    launches[g_tm.kid[i]] += 1;
  }
  g_tm.used = 0;
  return 0;
}

size_t ltc_preamble_workspace_bytes(int64_t rows, int32_t D) {
  int err = 0;
  const DeviceInfo di = device_info(&err);
  if (err || rows < 1 || D < 1) return 0;
  return (size_t)preamble_blocks(rows, di.sms) * 4 * D * sizeof(float);
}

int ltc_preamble_forward(int64_t rows, int32_t D, float eps, const float* x, const float* ln_w,
                         const float* ln_b, const float* in_w, const float* in_b, float* y, float* stats,
                         ltc_stream_t stream) {
  if (rows < 1 || D < 1 || D > 1024) return fail("ltc_preamble_forward: need rows >= 1 and 1 <= D <= 1024");
  if (!x || !ln_w || !ln_b || !in_w || !in_b || !y || !stats) return fail("ltc_preamble_forward: NULL pointer");
  int err = 0;
  const DeviceInfo di = device_info(&err);
  if (err) return 1;
  PreambleArgs a{};
  a.x = x; a.ln_w = ln_w; a.ln_b = ln_b; a.in_w = in_w; a.in_b = in_b; a.y = y; a.stats = stats;
  a.rows = rows; a.D = D; a.eps = eps;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  {
    TimedLaunch tl(LTC_KERNEL_PREAMBLE_FWD, st);
    e = launch_preamble_fwd(a, di.sms, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "preamble_fwd");
  g_last_error.clear();
  return 0;
}

int ltc_preamble_backward(int64_t rows, int32_t D, const float* x, const float* dy, const float* ln_w,
                          const float* ln_b, const float* in_w, const float* stats, float* dx, float* g_ln_w,
                          float* g_ln_b, float* g_in_w, float* g_in_b, void* workspace, size_t workspace_bytes,
                          ltc_stream_t stream) {
  if (rows < 1 || D < 1 || D > 1024) return fail("ltc_preamble_backward: need rows >= 1 and 1 <= D <= 1024");
  if (!x || !dy || !ln_w || !ln_b || !in_w || !stats || !dx || !g_ln_w || !g_ln_b || !g_in_w || !g_in_b ||
      !workspace)
    return fail("ltc_preamble_backward: NULL pointer");
  int err = 0;
  const DeviceInfo di = device_info(&err);
  if (err) return 1;
  const size_t need = (size_t)preamble_blocks(rows, di.sms) * 4 * D * sizeof(float);
  if (workspace_bytes < need)
    return fail("ltc_preamble_backward: workspace of %zu bytes is smaller than the %zu bytes required",
                workspace_bytes, need);
  PreambleArgs a{};
  a.x = x; a.dy = dy; a.ln_w = ln_w; a.ln_b = ln_b; a.in_w = in_w; a.stats = const_cast<float*>(stats); a.dx = dx;
  a.part = static_cast<float*>(workspace);
  a.g_in_w = g_in_w; a.g_in_b = g_in_b; a.g_ln_w = g_ln_w; a.g_ln_b = g_ln_b;
  a.rows = rows; a.D = D;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  {
    TimedLaunch tl(LTC_KERNEL_PREAMBLE_BWD, st);
    e = launch_preamble_bwd(a, di.sms, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "preamble_bwd");
  g_last_error.clear();
  return 0;
}

int ltc_checked_build(void) { return (int)ltc::check_readers().size(); }

int ltc_check_errors(int* count, int* first_site) {
  if (!count || !first_site) return fail("ltc_check_errors: NULL output");
  *count = 0;
  *first_site = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  for (auto r : ltc::check_readers())
    if (r(count, first_site) != 0) return -1;
  return 0;
}

int ltc_wait_timeouts(void) {
  int n = 0, m = 0;
  if (ltc::read_wait_timeouts(&n) != 0 || ltc::read_stream_wait_timeouts(&m) != 0) return -1;
  return n + m;
}

int64_t ltc_launch_count(void) {
  std::lock_guard<std::mutex> lk(g_tm_mu);
  return g_tm.launches;
}

int ltc_plan(const LtcDims* dims, LtcPlan* out) {
  Layout L;
  DeviceInfo di;
  if (!out) return fail("out is NULL");
  if (make_layout(dims, &L, &di)) return 1;
  FwdBuffers fb;
  BwdBuffers bb;
  out->saved_bytes = (L.saved_floats_v + L.saved_floats_r) * sizeof(float) + 256;
  out->fwd_workspace_bytes = carve_fwd(dims, L, nullptr, &fb);
  out->bwd_workspace_bytes = carve_bwd(dims, L, nullptr, &bb);
  out->wide = L.rp.wide ? 1 : 0;
  out->padded_h = L.rp.HP;
  out->fwd_ctas = L.rp.grid_fwd;
  out->bwd_ctas = L.rp.grid_bwd;
  out->lean_chunk_steps = L.lean ? L.tc : 0;
  g_last_error.clear();
  return 0;
}

int ltc_forward(const LtcDims* dims, const LtcParams* params, const float* x, const float* h0, float* outputs,
                float* h_final, void* saved, void* workspace, size_t workspace_bytes, ltc_stream_t stream) {
  Layout L;
  DeviceInfo di;
  if (make_layout(dims, &L, &di) || check_params(params)) return 1;
  if (!x || !outputs || !h_final || !workspace) return fail("ltc_forward: NULL x/outputs/h_final/workspace");
  FwdBuffers b;
  const size_t need = carve_fwd(dims, L, nullptr, &b);
  if (workspace_bytes < need)
    return fail("ltc_forward: workspace of %zu bytes is smaller than the %zu bytes required", workspace_bytes,
                need);
  carve_fwd(dims, L, workspace, &b);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int HP = L.rp.HP;

  PackArgs pa = pack_args(dims, params, HP);
  pa.pack = b.pack; pa.packT = nullptr; pa.spack = b.spack; pa.nrn = b.nrn;
  cudaError_t e;
  {
    TimedLaunch tl(LTC_KERNEL_PACK_FWD, st);
    e = launch_pack(pa, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "pack");
  if (L.rp.sparse) {
    TimedLaunch tl(LTC_KERNEL_PACK_FWD, st);
    e = launch_build_slots(pa, b.tables, st);
    if (e != cudaSuccess) return cuda_fail(e, "build_slots");
  }
  if (L.skip_sens) {
    TimedLaunch tl(LTC_KERNEL_PACK_FWD, st);
    e = launch_build_sens(pa, b.stables, st);
    if (e != cudaSuccess) return cuda_fail(e, "build_sens");
  }

  SensFwdArgs sa{};
  sa.spack = b.spack; sa.x = x; sa.sn = b.sn; sa.sd = b.sd; sa.rows = L.rows;
  sa.D = dims->D; sa.H = dims->H; sa.HP = HP;
  {
    TimedLaunch tl(LTC_KERNEL_SENSORY_FWD, st);
    e = L.skip_sens ? launch_sensory_fwd_sparse(sa, b.stables, di.sms, st) : launch_sensory_fwd(sa, di.sms, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "sensory_fwd");

  RecFwdArgs ra{};
  ra.pack = b.pack; ra.nrn = b.nrn; ra.sn = b.sn; ra.sd = b.sd; ra.h0 = h0;
  ra.out = outputs; ra.hT = h_final;
  if (saved && !L.lean) {
    Carver c(saved);
    ra.V = c.take<float>(L.saved_floats_v);
    ra.R = c.take<float>(L.saved_floats_r);
  }
  ra.B = dims->B; ra.T = dims->T; ra.H = dims->H; ra.U = dims->ode_unfolds; ra.HP = HP;
  ra.ns = L.rp.ns_fwd; ra.eps = dims->epsilon; ra.scratch = b.scratch; ra.tables = b.tables;
  {
    TimedLaunch tl(LTC_KERNEL_RECURRENT_FWD, st);
    e = launch_recurrent_fwd(ra, L.rp, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "recurrent_fwd");
  if (saved && L.lean) {  // step-boundary states: h0, then the outputs
    Carver c(saved);
    float* ck = c.take<float>(L.saved_floats_v);
    const size_t bh = (size_t)dims->B * dims->H * sizeof(float);
    e = h0 ? cudaMemcpyAsync(ck, h0, bh, cudaMemcpyDeviceToDevice, st) : cudaMemsetAsync(ck, 0, bh, st);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(ck + (size_t)dims->B * dims->H, outputs, bh * dims->T, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "lean checkpoint copy");
  }
  g_last_error.clear();
  return 0;
}

int ltc_backward(const LtcDims* dims, const LtcParams* params, const float* x, const void* saved,
                 const float* grad_outputs, const int64_t go_strides[3], const float* grad_state,
                 const LtcGrads* grads, void* workspace, size_t workspace_bytes, ltc_stream_t stream) {
  Layout L;
  DeviceInfo di;
  if (make_layout(dims, &L, &di) || check_params(params)) return 1;
  if (!x || !saved || !grad_outputs || !go_strides || !grads || !workspace)
    return fail("ltc_backward: NULL x/saved/grad_outputs/go_strides/grads/workspace");
  const float* gp[] = {grads->x_seq, grads->state, grads->w_pos, grads->w_erev, grads->mu, grads->sigma,
                       grads->sensory_mu, grads->sensory_sigma, grads->sensory_erev, grads->sensory_w_pos,
                       grads->cm_t, grads->gleak_pos, grads->vleak};
  for (const float* q : gp)
    if (!q) return fail("ltc_backward: a gradient output pointer is NULL");
  BwdBuffers b;
  const size_t need = carve_bwd(dims, L, nullptr, &b);
  if (workspace_bytes < need)
    return fail("ltc_backward: workspace of %zu bytes is smaller than the %zu bytes required", workspace_bytes,
                need);
  carve_bwd(dims, L, workspace, &b);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int HP = L.rp.HP;

  PackArgs pa = pack_args(dims, params, HP);
  pa.pack = b.pack; pa.packT = b.packT; pa.spack = b.spack; pa.nrn = b.nrn;
  pa.packT_qc = stream_chunk_cols(L.rp);
  cudaError_t e;
  {
    TimedLaunch tl(LTC_KERNEL_PACK_BWD, st);
    e = launch_pack(pa, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "pack");
  if (L.rp.sparse) {
    TimedLaunch tl(LTC_KERNEL_PACK_BWD, st);
    e = launch_build_slots(pa, b.tables, st);
    if (e != cudaSuccess) return cuda_fail(e, "build_slots");
  }
  if (b.stables) {
    TimedLaunch tl(LTC_KERNEL_PACK_BWD, st);
    e = launch_build_sens(pa, b.stables, st);
    if (e != cudaSuccess) return cuda_fail(e, "build_sens");
  }
  if (b.sbtables) {
    TimedLaunch tl(LTC_KERNEL_PACK_BWD, st);
    e = launch_build_sens_slots(pa, b.sbtables, st);
    if (e != cudaSuccess) return cuda_fail(e, "build_sens_slots");
  }

  Carver sc(const_cast<void*>(saved));
  RecBwdArgs ra{};
  ra.pack = b.pack; ra.packT = b.packT; ra.nrn = b.nrn;
  ra.gout = grad_outputs; ra.go_sb = go_strides[0]; ra.go_st = go_strides[1]; ra.go_sh = go_strides[2];
  ra.gstate = grad_state; ra.gsn = b.gsn; ra.gsd = b.gsd; ra.gh0 = grads->state;
  ra.part = b.rpart; ra.partn = b.rpartn;
  ra.B = dims->B; ra.T = dims->T; ra.H = dims->H; ra.U = dims->ode_unfolds; ra.HP = HP;
  ra.ns = L.rp.ns_bwd; ra.scratch = b.scratch; ra.tables = b.tables;
  if (!L.lean) {
    ra.V = sc.take<float>(L.saved_floats_v);
    ra.R = sc.take<float>(L.saved_floats_r);
    {
      TimedLaunch tl(LTC_KERNEL_RECURRENT_BWD, st);
      e = launch_recurrent_bwd(ra, L.rp, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "recurrent_bwd");
  } else if (int rc = lean_recurrent_backward(dims, L, di, b, sc.take<float>(L.saved_floats_v), x, ra, st)) {
    return rc;
  }

  SensBwdArgs sa{};
  sa.spack = b.spack; sa.x = x; sa.gsn = b.gsn; sa.gsd = b.gsd; sa.dx = grads->x_seq;
  sa.part = b.spart; sa.rows = L.rows; sa.D = dims->D; sa.H = dims->H; sa.HP = HP; sa.nsplit = L.sp.nsplit;
  {
    TimedLaunch tl(LTC_KERNEL_SENSORY_BWD, st);
    e = L.skip_sens_bwd ? launch_sensory_bwd_sparse(sa, L.sp, b.sbtables, b.dxpart, st)
                        : launch_sensory_bwd(sa, L.sp, b.dxpart, L.rp.tanh_space, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "sensory_bwd");

  FinishArgs fa{};
  fa.rec_part = b.rpart; fa.rec_partn = b.rpartn; fa.rslots = L.rp.slots_bwd; fa.rec_transposed = L.rp.wide && !L.rp.streamed;
  fa.rec_tanh_space = L.rp.tanh_space;
  if (L.rp.sparse) {
    fa.skip_w_pos = params->w_pos;
    fa.skip_w_erev = params->w_erev;
  }
  if (L.skip_sens_bwd) fa.skip_sw = params->sensory_w_pos;
  fa.sens_part = b.spart; fa.nsplit = L.sp.nsplit; fa.dxpart = b.dxpart; fa.nqc = L.sp.nqc; fa.rows = L.rows;
  fa.mu = params->mu; fa.sigma = params->sigma; fa.smu = params->sensory_mu; fa.ssig = params->sensory_sigma;
  fa.serev = params->sensory_erev; fa.sw = params->sensory_w_pos;
  fa.g_w_pos = grads->w_pos; fa.g_w_erev = grads->w_erev; fa.g_mu = grads->mu; fa.g_sigma = grads->sigma;
  fa.g_smu = grads->sensory_mu; fa.g_ssig = grads->sensory_sigma; fa.g_serev = grads->sensory_erev;
  fa.g_sw = grads->sensory_w_pos; fa.g_cm = grads->cm_t; fa.g_gl = grads->gleak_pos; fa.g_vl = grads->vleak;
  fa.g_x = grads->x_seq; fa.D = dims->D; fa.H = dims->H; fa.HP = HP;
  {
    TimedLaunch tl(LTC_KERNEL_FINISH, st);
    e = launch_finish(fa, di.sms, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "finish");
  g_last_error.clear();
  return 0;
}

}  // extern "C"

namespace {
// Lean backward of the recurrent part: segments of L.tc steps, newest first.  For
// each: stage its x rows and start state, recompute its sensory sums and unfolds
// (V, R) with the forward kernels, run the recurrent backward over it (adjoint in
// from the newer segment, parameter partials accumulated), and scatter its g_sn,
// g_sd rows into the full buffers the sensory backward reads.
int lean_recurrent_backward(const LtcDims* dims, const Layout& L, const DeviceInfo& di, const BwdBuffers& b,
                            const float* ck, const float* x, RecBwdArgs ra, cudaStream_t st) {
  const int B = dims->B, T = dims->T, D = dims->D, H = dims->H, HP = L.rp.HP;
  const size_t f4 = sizeof(float);
  const float* gin = ra.gstate;  // dL/d(state at the segment's end)
  float* gbuf[2] = {b.ghA, b.ghB};
  int gsel = 0;
  cudaError_t e = cudaSuccess;
  const int nseg = (T + L.tc - 1) / L.tc;
  for (int seg = nseg - 1; seg >= 0; --seg) {
    const int t0 = seg * L.tc, tc = T - t0 < L.tc ? T - t0 : L.tc;
    // x rows (b, t0 .. t0+tc) -> (B*tc, D); the state at t0 -> (B, H)
    e = cudaMemcpy2DAsync(b.xc, (size_t)tc * D * f4, x + (size_t)t0 * D, (size_t)T * D * f4, (size_t)tc * D * f4,
                          B, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "lean: stage x");
    const float* h_start = ck;  // h0 block
    if (t0 > 0) {
      e = cudaMemcpy2DAsync(b.hs, (size_t)H * f4, ck + (size_t)B * H + (size_t)(t0 - 1) * H, (size_t)T * H * f4,
                            (size_t)H * f4, B, cudaMemcpyDeviceToDevice, st);
      if (e != cudaSuccess) return cuda_fail(e, "lean: stage state");
      h_start = b.hs;
    }
    SensFwdArgs sa{};
    sa.spack = b.spack; sa.x = b.xc; sa.sn = b.snc; sa.sd = b.sdc; sa.rows = (long long)B * tc;
    sa.D = D; sa.H = H; sa.HP = HP;
    {
      TimedLaunch tl(LTC_KERNEL_SENSORY_FWD, st);
      e = b.stables ? launch_sensory_fwd_sparse(sa, b.stables, di.sms, st) : launch_sensory_fwd(sa, di.sms, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "lean: sensory_fwd");
    RecFwdArgs fa{};
    fa.pack = b.pack; fa.nrn = b.nrn; fa.sn = b.snc; fa.sd = b.sdc; fa.h0 = h_start;
    fa.out = nullptr; fa.hT = nullptr; fa.V = b.Vc; fa.R = b.Rc;
    fa.B = B; fa.T = tc; fa.H = H; fa.U = dims->ode_unfolds; fa.HP = HP;
    fa.ns = L.rp.ns_fwd; fa.eps = dims->epsilon; fa.scratch = b.fscratch; fa.tables = b.tables;
    {
      TimedLaunch tl(LTC_KERNEL_RECURRENT_FWD, st);
      e = launch_recurrent_fwd(fa, L.rp, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "lean: recurrent_fwd");
    RecBwdArgs sb = ra;
    sb.V = b.Vc; sb.R = b.Rc; sb.T = tc;
    sb.gout = ra.gout + (long long)t0 * ra.go_st;
    sb.gstate = gin;
    sb.gsn = b.gsnc; sb.gsd = b.gsdc;
    sb.gh0 = t0 == 0 ? ra.gh0 : gbuf[gsel];
    sb.accumulate = seg != nseg - 1;
    {
      TimedLaunch tl(LTC_KERNEL_RECURRENT_BWD, st);
      e = launch_recurrent_bwd(sb, L.rp, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "lean: recurrent_bwd");
    float* gfull[2] = {ra.gsn, ra.gsd};
    const float* gseg[2] = {b.gsnc, b.gsdc};
    for (int k = 0; k < 2; ++k) {
      e = cudaMemcpy2DAsync(gfull[k] + (size_t)t0 * H, (size_t)T * H * f4, gseg[k], (size_t)tc * H * f4,
                            (size_t)tc * H * f4, B, cudaMemcpyDeviceToDevice, st);
      if (e != cudaSuccess) return cuda_fail(e, "lean: scatter g_sn/g_sd");
    }
    gin = sb.gh0;
    gsel ^= 1;
  }
  return 0;
}
}  // namespace

// ---------------------------------------------------------------------------
// Step-level calls: the reference's per-step exports (csrc/ltc_kernels.cu:675-950),
// built from the same kernels with T = 1.
// ---------------------------------------------------------------------------
namespace {

int step_layout(const LtcDims* d, int kind, Layout* L, DeviceInfo* di) {
  if (!d) return fail("dims is NULL");
  if (d->B < 1 || d->H < 1 || d->H > 512) return fail("invalid step dims: B=%d H=%d", d->B, d->H);
  if ((kind == 0 || kind == 2) && d->D < 1) return fail("invalid step dims: D=%d", d->D);
  if ((kind == 1 || kind == 3) && d->ode_unfolds < 1) return fail("invalid step dims: ode_unfolds=%d", d->ode_unfolds);
  int err = 0;
  *di = device_info(&err);
  if (err) return 1;
  if (di->major != 10) return fail("libltc_sm100 requires an sm_100 (B200-class) GPU");
  L->rp = plan_recurrent(d->B, d->H, di->sms, d->flags & LTC_FLAG_FORCE_WIDE);
  L->rows = d->B;
  L->sp = plan_sensory_bwd(L->rows, d->D > 0 ? d->D : 1, L->rp.HP, di->sms);
  L->saved_floats_v = (size_t)(d->ode_unfolds + 1) * d->B * d->H;
  L->saved_floats_r = (size_t)d->ode_unfolds * d->B * d->H;
  return 0;
}

struct StepBuffers {
  float4 *pack, *packT, *spack, *nrn;
  float *V, *R, *out, *rpart, *rpartn, *spart, *dxpart, *scratch_f, *scratch_b;
};

size_t carve_step(const LtcDims* d, const Layout& L, int kind, void* ws, StepBuffers* b) {
  Carver c(ws);
  const int HP = L.rp.HP;
  *b = StepBuffers{};
  if (kind == 0 || kind == 2) b->spack = c.take<float4>((size_t)d->D * HP);
  if (kind == 1 || kind == 3) {
    b->pack = c.take<float4>((size_t)HP * HP);
    b->nrn = c.take<float4>(HP);
    b->V = c.take<float>(L.saved_floats_v);
    b->R = c.take<float>(L.saved_floats_r);
    b->out = c.take<float>((size_t)d->B * d->H);
    b->scratch_f = L.rp.scratch_fwd ? c.take<float>(L.rp.scratch_fwd) : nullptr;
  }
  if (kind == 3) {
    b->packT = c.take<float4>((size_t)HP * HP);
    b->rpart = c.take<float>((size_t)L.rp.slots_bwd * 4 * HP * HP);
    b->rpartn = c.take<float>((size_t)L.rp.slots_bwd * 5 * HP);
    b->scratch_b = L.rp.scratch_bwd ? c.take<float>(L.rp.scratch_bwd) : nullptr;
  }
  if (kind == 2) {
    b->spart = c.take<float>(L.sp.part_floats);
    b->dxpart = L.sp.dxpart_floats ? c.take<float>(L.sp.dxpart_floats) : nullptr;
  }
  return c.off + 256;
}

int step_begin(const LtcDims* d, int kind, void* ws, size_t wsb, Layout* L, DeviceInfo* di, StepBuffers* b) {
  if (step_layout(d, kind, L, di)) return 1;
  const size_t need = carve_step(d, *L, kind, nullptr, b);
  if (!ws || wsb < need) return fail("step call: workspace of %zu bytes is smaller than the %zu bytes required", wsb, need);
  carve_step(d, *L, kind, ws, b);
  return 0;
}

// recurrent forward of one step (T = 1) from `state`, saving V/R in the workspace
cudaError_t step_unfold_fwd(const LtcDims* d, const LtcParams* p, const Layout& L, const DeviceInfo& di,
                            const StepBuffers& b, const float* state, const float* wn, const float* wd,
                            cudaStream_t st) {
  PackArgs pa = pack_args(d, p, L.rp.HP);
  pa.ssig = nullptr;  // recurrent + per-neuron packs only
  pa.pack = b.pack; pa.packT = b.packT; pa.nrn = b.nrn;
  pa.packT_qc = stream_chunk_cols(L.rp);
  cudaError_t e = launch_pack(pa, st);
  if (e != cudaSuccess) return e;
  RecFwdArgs ra{};
  ra.pack = b.pack; ra.nrn = b.nrn; ra.sn = wn; ra.sd = wd; ra.h0 = state;
  // the final state is written twice with identical values (out after the last
  // unfold, hT after the loop, by different threads): both go to b.out
  ra.out = b.out; ra.hT = b.out;
  ra.V = b.V; ra.R = b.R;
  ra.B = d->B; ra.T = 1; ra.H = d->H; ra.U = d->ode_unfolds; ra.HP = L.rp.HP;
  ra.ns = L.rp.ns_fwd; ra.eps = d->epsilon; ra.scratch = b.scratch_f;
  (void)di;
  return launch_recurrent_fwd(ra, L.rp, st);
}

}  // namespace

extern "C" {

int ltc_step_workspace_bytes(const LtcDims* dims, int kind, size_t* bytes) {
  Layout L;
  DeviceInfo di;
  StepBuffers b;
  if (!bytes) return fail("bytes is NULL");
  if (kind < 0 || kind > 3) return fail("kind must be 0..3");
  if (step_layout(dims, kind, &L, &di)) return 1;
  *bytes = carve_step(dims, L, kind, nullptr, &b);
  g_last_error.clear();
  return 0;
}

int ltc_step_sensory_forward(const LtcDims* dims, const LtcParams* params, const float* inputs, float* w_num,
                             float* w_den, void* workspace, size_t workspace_bytes, ltc_stream_t stream) {
  Layout L; DeviceInfo di; StepBuffers b;
  if (step_begin(dims, 0, workspace, workspace_bytes, &L, &di, &b)) return 1;
  if (!params || !params->sensory_sigma || !params->sensory_mu || !params->sensory_w_pos || !params->sensory_erev ||
      !inputs || !w_num || !w_den)
    return fail("ltc_step_sensory_forward: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  PackArgs pa = pack_args(dims, params, L.rp.HP);
  pa.w_pos = nullptr; pa.cm = nullptr;  // sensory pack only
  pa.spack = b.spack;
  cudaError_t e = launch_pack(pa, st);
  if (e == cudaSuccess) {
    SensFwdArgs sa{};
    sa.spack = b.spack; sa.x = inputs; sa.sn = w_num; sa.sd = w_den; sa.rows = dims->B;
    sa.D = dims->D; sa.H = dims->H; sa.HP = L.rp.HP;
    e = launch_sensory_fwd(sa, di.sms, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "ltc_step_sensory_forward");
  g_last_error.clear();
  return 0;
}

int ltc_step_unfold_forward(const LtcDims* dims, const LtcParams* params, const float* state, const float* w_num,
                            const float* w_den, float* state_out, float* v_buffer, void* workspace,
                            size_t workspace_bytes, ltc_stream_t stream) {
  Layout L; DeviceInfo di; StepBuffers b;
  if (step_begin(dims, 1, workspace, workspace_bytes, &L, &di, &b)) return 1;
  if (!params || !params->w_pos || !params->w_erev || !params->mu || !params->sigma || !params->cm_t ||
      !params->gleak_pos || !params->vleak || !state || !w_num || !w_den || !state_out)
    return fail("ltc_step_unfold_forward: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = step_unfold_fwd(dims, params, L, di, b, state, w_num, w_den, st);
  const size_t bh = (size_t)dims->B * dims->H * sizeof(float);
  if (e == cudaSuccess) e = cudaMemcpyAsync(state_out, b.out, bh, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && v_buffer)
    e = cudaMemcpyAsync(v_buffer, b.V, bh * dims->ode_unfolds, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return cuda_fail(e, "ltc_step_unfold_forward");
  g_last_error.clear();
  return 0;
}

int ltc_step_sensory_backward(const LtcDims* dims, const LtcParams* params, const float* grad_w_num,
                              const float* grad_w_den, const float* inputs, float* grad_inputs, float* g_sigma,
                              float* g_mu, float* g_w_pos, float* g_erev, void* workspace, size_t workspace_bytes,
                              ltc_stream_t stream) {
  Layout L; DeviceInfo di; StepBuffers b;
  if (step_begin(dims, 2, workspace, workspace_bytes, &L, &di, &b)) return 1;
  if (!params || !params->sensory_sigma || !params->sensory_mu || !params->sensory_w_pos || !params->sensory_erev ||
      !grad_w_num || !grad_w_den || !inputs || !grad_inputs || !g_sigma || !g_mu || !g_w_pos || !g_erev)
    return fail("ltc_step_sensory_backward: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  PackArgs pa = pack_args(dims, params, L.rp.HP);
  pa.w_pos = nullptr; pa.cm = nullptr;
  pa.spack = b.spack;
  cudaError_t e = launch_pack(pa, st);
  if (e == cudaSuccess) {
    SensBwdArgs sa{};
    sa.spack = b.spack; sa.x = inputs; sa.gsn = grad_w_num; sa.gsd = grad_w_den; sa.dx = grad_inputs;
    sa.part = b.spart; sa.rows = dims->B; sa.D = dims->D; sa.H = dims->H; sa.HP = L.rp.HP; sa.nsplit = L.sp.nsplit;
    e = launch_sensory_bwd(sa, L.sp, b.dxpart, false, st);
  }
  if (e == cudaSuccess) {
    FinishArgs fa{};
    fa.sens_part = b.spart; fa.nsplit = L.sp.nsplit; fa.dxpart = b.dxpart; fa.nqc = L.sp.nqc; fa.rows = dims->B;
    fa.smu = params->sensory_mu; fa.ssig = params->sensory_sigma; fa.serev = params->sensory_erev;
    fa.sw = params->sensory_w_pos;
    fa.g_smu = g_mu; fa.g_ssig = g_sigma; fa.g_serev = g_erev; fa.g_sw = g_w_pos; fa.g_x = grad_inputs;
    fa.D = dims->D; fa.H = dims->H; fa.HP = L.rp.HP;
    e = launch_finish(fa, di.sms, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "ltc_step_sensory_backward");
  g_last_error.clear();
  return 0;
}

int ltc_step_unfold_backward(const LtcDims* dims, const LtcParams* params, const float* v_buffer, const float* w_num,
                             const float* w_den, const float* grad_output, float* grad_v, float* grad_w_num,
                             float* grad_w_den, float* g_w_pos, float* g_w_erev, float* g_mu, float* g_sigma,
                             float* g_cm, float* g_gleak, float* g_vleak, void* workspace, size_t workspace_bytes,
                             ltc_stream_t stream) {
  Layout L; DeviceInfo di; StepBuffers b;
  if (step_begin(dims, 3, workspace, workspace_bytes, &L, &di, &b)) return 1;
  if (!params || !params->w_pos || !params->w_erev || !params->mu || !params->sigma || !params->cm_t ||
      !params->gleak_pos || !params->vleak || !v_buffer || !w_num || !w_den || !grad_output || !grad_v ||
      !grad_w_num || !grad_w_den || !g_w_pos || !g_w_erev || !g_mu || !g_sigma || !g_cm || !g_gleak || !g_vleak)
    return fail("ltc_step_unfold_backward: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the reciprocal denominators are not part of the reference's v_buffer: recompute the
  // step's unfolds from its first state (v_buffer[0]) and keep V, R in the workspace
  cudaError_t e = step_unfold_fwd(dims, params, L, di, b, v_buffer, w_num, w_den, st);
  if (e == cudaSuccess) {
    RecBwdArgs ra{};
    ra.pack = b.pack; ra.packT = b.packT; ra.nrn = b.nrn; ra.V = b.V; ra.R = b.R;
    ra.gout = grad_output; ra.go_sb = dims->H; ra.go_st = 0; ra.go_sh = 1; ra.gstate = nullptr;
    ra.gsn = grad_w_num; ra.gsd = grad_w_den; ra.gh0 = grad_v; ra.part = b.rpart; ra.partn = b.rpartn;
    ra.B = dims->B; ra.T = 1; ra.H = dims->H; ra.U = dims->ode_unfolds; ra.HP = L.rp.HP; ra.ns = L.rp.ns_bwd;
    ra.scratch = b.scratch_b;
    e = launch_recurrent_bwd(ra, L.rp, st);
  }
  if (e == cudaSuccess) {
    FinishArgs fa{};
    fa.rec_part = b.rpart; fa.rec_partn = b.rpartn; fa.rslots = L.rp.slots_bwd;
    fa.rec_transposed = L.rp.wide && !L.rp.streamed; fa.rec_tanh_space = L.rp.tanh_space;
    fa.mu = params->mu; fa.sigma = params->sigma;
    fa.g_w_pos = g_w_pos; fa.g_w_erev = g_w_erev; fa.g_mu = g_mu; fa.g_sigma = g_sigma;
    fa.g_cm = g_cm; fa.g_gl = g_gleak; fa.g_vl = g_vleak; fa.D = 0; fa.H = dims->H; fa.HP = L.rp.HP; fa.nqc = 1;
    e = launch_finish(fa, di.sms, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "ltc_step_unfold_backward");
  g_last_error.clear();
  return 0;
}

}  // extern "C"
